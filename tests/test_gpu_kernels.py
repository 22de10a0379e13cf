"""GPU parity of every kernel against the CPU oracle, through the C ABI.

Bit-exact where the arithmetic allows it (LUT build, ordered apply, dequant,
encoder, route given the same logits); fp32-accumulation tolerance for the
bandwidth kernels, whose summation order differs from the reference's.
"""
import numpy as np
import pytest
import torch

from warp_b200 import container as C

pytestmark = pytest.mark.gpu

# The bandwidth kernels sum in another order than the reference; fp32 sums of
# a few thousand terms agree to ~1e-6 relative.  FFN outputs must stay within
# the path's 2e-3 relative-L2 contract.
TOL_KERNEL = 2e-5
TOL_FFN = 2e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _books(rng, n=9):
    return rng.uniform(-0.3, 0.3, (n, 256, 8)).astype(np.float16).view(np.uint16)


@pytest.mark.parametrize("nv", [16, 37, 288, 896])
def test_lut_build_bitexact(cuda, oracle, nv):
    from warp_b200 import ops
    rng = np.random.default_rng(nv)
    books, booksT = oracle.books_decode(_books(rng))
    x = rng.standard_normal(nv * 8).astype(np.float32)
    dT = torch.from_numpy(booksT).to(cuda)
    dx = torch.from_numpy(x).to(cuda)
    for cb in (0, 3, 6):
        got = ops.vq_build_lut(dT, dx, cb).cpu().numpy()
        want = oracle.lut_build(booksT, x, cb)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("M,nv", [(64, 16), (96, 16), (1024, 288), (2304, 128), (200, 40),
                                  (2048, 896)])
def test_vq_apply(cuda, oracle, M, nv):
    from warp_b200 import ops
    rng = np.random.default_rng(M * 7 + nv)
    idx = rng.integers(0, 256, C.index_bytes(M, nv * 8), dtype=np.uint8)
    scale = rng.uniform(0.01, 0.05, M).astype(np.float16).view(np.uint16)
    lut = rng.standard_normal((nv, 3, 256)).astype(np.float32)
    want = oracle.vq_rows(idx, scale, lut, M)
    di = torch.from_numpy(idx).to(cuda)
    ds = torch.from_numpy(scale.view(np.int16)).to(cuda)
    dl = torch.from_numpy(lut).to(cuda)
    got_o = ops.vq_apply(di, ds, dl, M, ordered=True).cpu().numpy()
    np.testing.assert_array_equal(got_o.view(np.uint32), want.view(np.uint32))
    got_f = ops.vq_apply(di, ds, dl, M, ordered=False).cpu().numpy()
    assert rel_l2(got_f, want) < TOL_KERNEL
    np.testing.assert_allclose(got_f, want, rtol=1e-4, atol=1e-5 * np.abs(want).max())


@pytest.mark.parametrize("M,N", [(96, 128), (1024, 2304), (2304, 1024)])
def test_vq_dequant_bitexact(cuda, oracle, M, N):
    from warp_b200 import ops
    rng = np.random.default_rng(M + N)
    books, _ = oracle.books_decode(_books(rng))
    idx = rng.integers(0, 256, C.index_bytes(M, N), dtype=np.uint8)
    scale = rng.uniform(0.01, 0.05, M).astype(np.float16).view(np.uint16)
    for cb in (0, 6):
        want = oracle.vq_dequant(idx, scale, books, M, N, cb)
        got = ops.vq_dequant(torch.from_numpy(idx).to(cuda),
                             torch.from_numpy(scale.view(np.int16)).to(cuda),
                             torch.from_numpy(books).to(cuda), M, N, cb).cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def test_vq_encode_bitexact(cuda, oracle):
    from warp_b200 import ops
    rng = np.random.default_rng(5)
    books = (rng.standard_normal((3, 256, 8)) * np.float32([[[1]], [[0.3]], [[0.1]]])).astype(np.float32)
    X = rng.standard_normal((20000, 8)).astype(np.float32)
    X /= np.abs(X).max(1, keepdims=True)
    X[:10] = books[0, :10]
    X[10] = 0.0
    want = oracle.vq_encode(X, books)
    got = ops.vq_encode(torch.from_numpy(X).to(cuda), torch.from_numpy(books).to(cuda))
    np.testing.assert_array_equal(got.cpu().numpy(), want)


def test_qwen_route_bitexact(cuda, oracle):
    from warp_b200 import ops
    rng = np.random.default_rng(11)
    for trial in range(200):
        E = int(rng.choice([8, 32, 64, 256, 384]))
        K = int(rng.integers(1, min(E, 16) + 1))
        T = int(rng.integers(1, 5))
        logits = (rng.standard_normal((T, E)) * float(rng.choice([0.1, 1, 5]))).astype(np.float32)
        if trial % 5 == 0:
            logits[:, rng.integers(0, E, E // 2)] = logits[:, :1]
        renorm = bool(trial % 2)
        idx, w = ops.qwen_moe_route(torch.from_numpy(logits).to(cuda), K, renorm)
        idx, w = idx.cpu().numpy(), w.cpu().numpy()
        for t in range(T):
            rc, ridx, rw = oracle.qwen_route(logits[t], K, renorm)
            np.testing.assert_array_equal(idx[t], ridx)
            # the softmax sum is a tree on the device and sequential in the
            # reference, and exp is correctly rounded on the device where
            # glibc's is within 0.502 ulp: weights agree to a few ulp, the
            # indices exactly
            np.testing.assert_allclose(w[t], rw, rtol=4e-6, atol=1e-7)


@pytest.mark.parametrize("func", [0, 1, 2])
def test_moe_route_matches_oracle(cuda, oracle, func):
    """moe_layer's router (model.c:5466-5556) on the device: scores, the
    selection-only bias, renorm with + 1e-20 and routed_scale.  Indices
    exactly, with ties forced (repeated logits; sigmoid saturated to 1.0);
    weights to an ulp (exp and log1p are rounded once from higher precision
    on the device, glibc's expf / log1pf are within about half an ulp)."""
    from warp_b200 import ops
    rng = np.random.default_rng(70 + func)
    for trial in range(120):
        E = int(rng.choice([8, 32, 64, 256, 384]))
        K = int(rng.integers(1, min(E, 16) + 1))
        T = int(rng.integers(1, 4))
        scale = float(rng.choice([0.1, 1.0, 5.0, 40.0]))
        logits = (rng.standard_normal((T, E)) * scale).astype(np.float32)
        if trial % 4 == 0:
            logits[:, rng.integers(0, E, E // 2)] = logits[:, :1]
        bias = None
        if trial % 3 == 0:
            bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
            if trial % 6 == 0:
                bias[rng.integers(0, E, E // 4)] = 0.0
        renorm = bool(trial % 2)
        rs = float(rng.choice([1.0, 2.5]))
        idx, w = ops.moe_route(torch.from_numpy(logits).to(cuda), K, func,
                               None if bias is None else torch.from_numpy(bias).to(cuda),
                               renorm, rs)
        idx, w = idx.cpu().numpy(), w.cpu().numpy()
        for t in range(T):
            rc, ridx, rw, _ = oracle.route_scored(logits[t], K, func, bias, renorm, rs)
            assert rc == 0
            np.testing.assert_array_equal(idx[t], ridx)
            np.testing.assert_allclose(w[t], rw, rtol=3e-7, atol=1e-30)


@pytest.mark.parametrize("bits,group", [(4, 32), (8, 0)])
@pytest.mark.parametrize("out,inn", [(2304, 2304), (512, 7168), (256, 18432)])
@pytest.mark.parametrize("batch,bf16", [(1, True), (1, False), (4, True), (16, True),
                                        (37, False), (64, True)])
def test_mvq_matvec(cuda, oracle, bits, group, out, inn, batch, bf16):
    from warp_b200 import ffi, ops, synth
    g = inn if group == 0 else group
    gen = torch.Generator(device="cpu").manual_seed(out + inn + bits)
    W = torch.randn(out, inn, generator=gen) * 0.02
    q, s = synth.quantize_q(W, g, bits)
    X = torch.randn(batch, inn, generator=gen)
    if bf16:
        X = X.to(torch.bfloat16)
    Xf = X.float().numpy()
    rowbytes = inn * bits // 8
    want = oracle.deq_matmul_f64(q.numpy(), s.numpy().view(np.uint16), Xf, out, inn, g,
                                 bits, rowbytes)
    got = ops.mvq_matvec(q.to(cuda), s.to(cuda), X.to(cuda), out, inn, g, bits).cpu().numpy()
    assert ffi.load().warp_mvq_status(1) == 0, ffi.load().warp_last_error()
    assert got.shape == want.shape
    assert rel_l2(got, want) < TOL_KERNEL, rel_l2(got, want)
    if batch == 1 and not bf16:
        port = oracle.mvq_rows(q.numpy(), s.numpy().view(np.uint16), Xf[0], out, inn, g,
                               bits, rowbytes)
        assert rel_l2(got[0], port) < TOL_KERNEL


@pytest.mark.parametrize("M,nv", [(64, 16), (200, 40), (2048, 896), (7168, 256)])
def test_vq4p_bitexact(cuda, oracle, M, nv):
    """VQ4P on the device: the int8 table of x (4 x 64 FMA-chain table, then
    vq_quant_lut) and waste_vq_rows_p6, bit for bit against the oracle."""
    from warp_b200 import ops
    rng = np.random.default_rng(M * 7 + nv)
    booksT = rng.uniform(-0.3, 0.3, (5, 8, 64)).astype(np.float32)
    x = (rng.standard_normal(nv * 8) * np.repeat(rng.uniform(0.01, 3.0, nv), 8)).astype(np.float32)
    q, ls = ops.vq4p_lut(torch.from_numpy(booksT).to(cuda), torch.from_numpy(x).to(cuda), 1)
    lut = oracle.lut_build_se(booksT, x, 1, 4, 64)
    wq, wls = oracle.vq_quant_lut(lut)
    np.testing.assert_array_equal(q.cpu().numpy(), wq)
    np.testing.assert_array_equal(ls.cpu().numpy().view(np.uint32), wls.view(np.uint32))
    idx = rng.integers(0, 256, ((M + 63) // 64) * nv * 64 * 3, dtype=np.uint8)
    scale = rng.uniform(0.01, 0.05, M).astype(np.float16).view(np.uint16)
    y = ops.vq4p_apply(torch.from_numpy(idx).to(cuda),
                       torch.from_numpy(scale.view(np.int16)).to(cuda), q, ls, M)
    want = oracle.vq_rows_p6(idx, scale, wq, wls, M)
    np.testing.assert_array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_mvq_matvec_batch_limits(cuda):
    """Batch 65 is refused (the engine's prefill chunk is 64 tokens); a
    smaller call after a larger one on the same stream reuses its scratch."""
    from warp_b200 import ffi, ops, synth
    W = torch.randn(64, 256) * 0.02
    q, s = synth.quantize_q(W, 32, 4)
    with pytest.raises(ffi.WarpError):
        ops.mvq_matvec(q.to(cuda), s.to(cuda), torch.randn(65, 256, device=cuda), 64, 256, 32, 4)
    X = torch.randn(64, 256, device=cuda)
    big = ops.mvq_matvec(q.to(cuda), s.to(cuda), X, 64, 256, 32, 4)
    small = ops.mvq_matvec(q.to(cuda), s.to(cuda), X[:5].contiguous(), 64, 256, 32, 4)
    torch.cuda.synchronize()
    assert torch.allclose(big[:5], small, rtol=1e-6, atol=1e-6)
