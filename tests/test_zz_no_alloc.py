"""warp_vq_apply_noalloc — the gather path with fixed module-scope scratch.

Some callers cannot allocate device memory while they run (an engine that
sizes all of HBM once at load, a context without a stream-ordered memory
pool, a decode loop that must not take an allocator lock); this entry point
serves them.  Checked through the C ABI against warp_vq_apply's bandwidth
path (ordered = 0) and against the oracle's vq_rows, on two calls in a row
with different shapes, so a stale error word or partials left by the first
call would show in the second.  The file name sorts last so it also runs
after every other GPU test in one session.
"""
import ctypes

import numpy as np
import pytest
import torch

from warp_b200 import container as C

pytestmark = pytest.mark.gpu

TOL_KERNEL = 2e-5        # same tolerance as the other bandwidth-kernel tests


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _case(rng, M, nv, dev):
    idx = rng.integers(0, 256, C.index_bytes(M, nv * 8), dtype=np.uint8)
    scale = rng.uniform(0.01, 0.05, M).astype(np.float16).view(np.uint16)
    lut = rng.standard_normal((nv, 3, 256)).astype(np.float32)
    return (torch.from_numpy(idx).to(dev), torch.from_numpy(scale.view(np.int16)).to(dev),
            torch.from_numpy(lut).to(dev))


def test_noalloc_matches_vq_apply_twice(cuda, oracle):
    from warp_b200 import ffi
    lib = ffi.load()
    rng = np.random.default_rng(2024)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for M, nv in ((2048, 896), (7168, 256)):
        di, ds, dl = _case(rng, M, nv, cuda)
        want = torch.empty(M, dtype=torch.float32, device=cuda)
        ffi.check(lib.warp_vq_apply(_p(want), _p(di), _p(ds), _p(dl), M, nv, 0, st))
        got = torch.full((M,), float("nan"), dtype=torch.float32, device=cuda)
        ffi.check(lib.warp_vq_apply_noalloc(_p(got), _p(di), _p(ds), _p(dl), M, nv, st))
        w, g = want.cpu().numpy(), got.cpu().numpy()
        assert np.isfinite(g).all()
        assert rel_l2(g, w) < TOL_KERNEL
        # and against the oracle's vq_rows on the same codes, scales and table
        o = oracle.vq_rows(di.cpu().numpy(), ds.cpu().numpy().view(np.uint16),
                           dl.cpu().numpy(), M)
        assert rel_l2(g, o) < TOL_KERNEL


def test_noalloc_rejects_oversize(cuda):
    from warp_b200 import ffi
    lib = ffi.load()
    rng = np.random.default_rng(7)
    di, ds, dl = _case(rng, 64, 896, cuda)
    y = torch.empty(64, dtype=torch.float32, device=cuda)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # 28 chunks of images (2.6 MiB) + 28 * 100000 * 4 bytes of partials is
    # above the fixed 8 MiB: refused before anything is launched.
    rc = lib.warp_vq_apply_noalloc(_p(y), _p(di), _p(ds), _p(dl), 100000, 896, st)
    assert rc == -1
    assert b"scratch" in lib.warp_last_error()
