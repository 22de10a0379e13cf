"""The tensor-core (tcgen05) prefill GEMMs against the oracle.

warp_vq_matmul computes Y = X W^T for a VQ3R matrix with fp16 operands and
fp32 accumulation. It is checked two ways:
* Against an fp64 emulation of exactly that rounding: the weights
  (C0 + C1) + C2 rounded once to fp16, X rounded to fp16, row scale applied
  after. This must agree to accumulation-order differences (1e-5), so any
  slip in a descriptor, a tile layout or the tensor-memory readout shows up.
* Against the fp32 reference path (vq_dequant, then the product). This must
  agree within the FFN contract of 2e-3 relative L2.
"""
import numpy as np
import pytest
import torch

from warp_b200 import container as C

pytestmark = pytest.mark.gpu

TOL_FFN = 2e-3
TOL_EMUL = 1e-5


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _books(rng, n=9):
    return rng.uniform(-0.3, 0.3, (n, 256, 8)).astype(np.float16).view(np.uint16)


def _emulated(oracle, idx, scale, books, M, N, cb, X):
    ones = np.full(M, 0x3C00, np.uint16)                      # fp16 1.0
    W = oracle.vq_dequant(idx, ones, books, M, N, cb)          # (C0 + C1) + C2, fp32
    W16 = W.astype(np.float16).astype(np.float64)
    X16 = X.astype(np.float16).astype(np.float64)
    s = scale.view(np.float16).astype(np.float64)
    return (X16 @ W16.T) * s[None, :]


@pytest.mark.parametrize("M,N,T", [(256, 512, 200), (300, 264, 64), (128, 64, 1),
                                   (2048, 7168, 130)])
def test_vq_matmul(cuda, oracle, M, N, T):
    from warp_b200 import ops
    rng = np.random.default_rng(M + N + T)
    books, _ = oracle.books_decode(_books(rng))
    idx = rng.integers(0, 256, C.index_bytes(M, N), dtype=np.uint8)
    scale = rng.uniform(0.01, 0.05, M).astype(np.float16).view(np.uint16)
    X = rng.standard_normal((T, N)).astype(np.float32)
    cb = 3
    Y = ops.vq_matmul(torch.from_numpy(X).to(cuda), torch.from_numpy(idx).to(cuda),
                      torch.from_numpy(scale.view(np.int16)).to(cuda),
                      torch.from_numpy(books).to(cuda), M, cb).cpu().numpy()
    ops.umma_status()
    want = X.astype(np.float64) @ oracle.vq_dequant(idx, scale, books, M, N, cb).T.astype(np.float64)
    emul = _emulated(oracle, idx, scale, books, M, N, cb, X)
    assert rel_l2(Y, emul) < TOL_EMUL
    assert rel_l2(Y, want) < TOL_FFN


@pytest.mark.parametrize("tile", [True, False])
@pytest.mark.parametrize("hidden,inter,E,K,T,gate", [
    (256, 128, 16, 4, 70, False),
    (384, 160, 8, 3, 200, True),           # partial chunks; experts with > 128 tokens
    (2304, 1024, 32, 8, 130, False),       # config 1 geometry
])
def test_moe_prefill(cuda, oracle, hidden, inter, E, K, T, gate, tile):
    """warp_moe_layer_prefill against the oracle's layer, token by token:
    routing exact, outputs within the FFN contract."""
    from test_gpu_moe import _layer, _oracle_layer
    layer = _layer(hidden, inter, E, hidden + T, True, gate, cuda)
    recs = layer.host_records()
    moe = layer.moe(K, tile_bank=tile, prefill_tokens=T)
    x = torch.randn(T, hidden, generator=torch.Generator().manual_seed(T)).to(cuda)
    out, idx, w = moe.prefill(x, want_route=True)
    moe.status()
    want, widx = _oracle_layer(oracle, layer, x.cpu().numpy(), K, True, True, recs)
    np.testing.assert_array_equal(idx.cpu().numpy(), widx)
    err = rel_l2(out.cpu().numpy(), want)
    assert err < TOL_FFN, err
    # the residual is added last
    res = torch.randn(T, hidden, generator=torch.Generator().manual_seed(T + 1)).to(cuda)
    out2 = moe.prefill(x, residual=res)
    torch.cuda.synchronize()
    assert torch.equal(out2, out + res)
    moe.close()


@pytest.mark.parametrize("bits,group,T", [(8, 32, 150), (8, 32, 65), (8, 32, 1)])
def test_moe_prefill_q8_shared(cuda, oracle, bits, group, T):
    """A Q8 g32 shared expert in prefill runs through the trunk matmul, 64
    tokens a launch (150 tokens: three launches, the last partial; 1 token:
    the CUDA-core path): routing exact, outputs within the FFN contract
    against the oracle."""
    from test_gpu_moe import _layer, _oracle_layer
    from warp_b200 import ffi
    hidden, inter, E, K = 384, 160, 8, 3
    layer = _layer(hidden, inter, E, 7 + T, True, True, cuda, bits=bits, group=group)
    recs = layer.host_records()
    moe = layer.moe(K, prefill_tokens=T)
    x = torch.randn(T, hidden, generator=torch.Generator().manual_seed(T + 3)).to(cuda)
    out, idx, w = moe.prefill(x, want_route=True)
    moe.status()
    assert ffi.load().warp_mvq_status(1) == 0
    want, widx = _oracle_layer(oracle, layer, x.cpu().numpy(), K, True, True, recs)
    np.testing.assert_array_equal(idx.cpu().numpy(), widx)
    err = rel_l2(out.cpu().numpy(), want)
    assert err < TOL_FFN, err
    moe.close()
