"""Host-side container layout and quantizers (CPU)."""
import numpy as np
import pytest
import torch

from warp_b200 import container as C


def test_record_layout_config1():
    g, u, d, s, end, rec = C.record_layout(2304, 1024)
    assert (g, end - C.HDR.size, rec) == (48, 2662912, 2666496)
    assert C.packed_bytes_per_expert(2304, 1024) == 2662912
    g, u, d, s, end, rec = C.record_layout(7168, 2048)
    assert end - C.HDR.size == 16537600


def test_block_roundtrip():
    rng = np.random.default_rng(0)
    for M, N in ((64, 16), (96, 128), (130, 64)):
        codes = rng.integers(0, 256, (M * N // 8, 3), dtype=np.uint8)
        b = C.block_indices(codes, M, N)
        assert b.size == C.index_bytes(M, N)
        np.testing.assert_array_equal(C.unblock_indices(b, M, N), codes)


def test_block_matches_oracle(oracle):
    rng = np.random.default_rng(1)
    M, N = 130, 64
    codes = rng.integers(0, 256, (M * N // 8, 3), dtype=np.uint8)
    np.testing.assert_array_equal(C.block_indices(codes, M, N), oracle.block_indices(codes, M, N))


def test_record_header_roundtrip():
    rng = np.random.default_rng(2)
    hidden, inter = 128, 64
    blocks = [rng.integers(0, 256, C.index_bytes(M, N), dtype=np.uint8)
              for M, N in ((inter, hidden), (inter, hidden), (hidden, inter))]
    scales = [rng.integers(0, 65535, n, dtype=np.uint16) for n in (inter, inter, hidden)]
    rec = C.write_record(3, 5, 9, blocks, scales, hidden, inter)
    assert len(rec) % 4096 == 0
    h = C.parse_header(rec)
    assert (h["magic"], h["layer"], h["expert_id"], h["fmt"], h["codebook_id"]) == \
        (C.MAGIC_EXPERT, 3, 5, 4, 9)
    assert h["rec_4k_blocks"] * 4096 == len(rec)


def test_codebook_roundtrip():
    rng = np.random.default_rng(3)
    b = rng.integers(0, 65535, (9, 256, 8), dtype=np.uint16)
    np.testing.assert_array_equal(C.parse_codebooks(C.codebook_bytes(b, 18)), b)


def test_quantizers_match_oracle(oracle):
    """quantize_q4g/q8g in torch (product) and in C (oracle) agree byte for
    byte, including the fp16 rounding of the scales."""
    from warp_b200 import synth
    gen = torch.Generator().manual_seed(0)
    W = torch.randn(64, 256, generator=gen) * 0.02
    W[3, :32] = 0.0
    for bits, g in ((4, 32), (8, 256), (4, 128)):
        q, s = synth.quantize_q(W, g, bits)
        oq, os_ = oracle.quant_q(W.numpy(), g, bits)
        np.testing.assert_array_equal(q.numpy().reshape(-1), oq)
        np.testing.assert_array_equal(s.numpy().view(np.uint16).reshape(-1), os_)
