"""The engine-facing boundary through the C ABI, with host pointers, the way
the reference engine calls it: waste_register_cuda on a waste_kernels table
(waste_backend.h:69-107), the mvq_rows_f32 slot with an mvq_arg (simd.h:35-39),
waste_cuda_vq3r with waste_vq_job batches (waste_metal.h:31-44), and the
release hook.  The "engine CPU kernel" here is a test fake computing with the
oracle; it only runs where the slot's contract says the CPU must."""
import ctypes

import numpy as np
import pytest

from warp_b200 import container as C

pytestmark = pytest.mark.gpu

TOL_KERNEL = 2e-5
P, I, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
SLOT = ctypes.CFUNCTYPE(None, I, I, P)
_KEEP = []          # the library keeps the fake CPU kernel's address for the process


class Kernels(ctypes.Structure):
    """waste_kernels (waste_backend.h:69-107)."""
    _fields_ = [("kda_step", P), ("short_conv_step", P), ("rmsnorm_gated", P),
                ("mvq_rows_f32", P), ("lutb_range", P), ("vq_rows_p6", P), ("vq_rows_e", P),
                ("on_device", I), ("mvq_rows_cpu", P), ("device_min_bytes", SZ)]


class MvqArg(ctypes.Structure):
    """mvq_arg (simd.h:35-39)."""
    _fields_ = [("y", P), ("W", P), ("ws", P), ("xq", P), ("xs", P), ("in_", I), ("ng", I),
                ("group", I), ("bits", I), ("rowbytes", SZ)]


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


class Engine:
    """A table as backend.c leaves it before the accelerator registers: the
    CPU kernel in mvq_rows_f32 and snapshotted into mvq_rows_cpu."""

    def __init__(self, oracle):
        self.oracle = oracle
        self.cpu_calls = 0
        self.mats = {}
        self.cpu = SLOT(self._cpu)
        self.t = Kernels()
        self.t.mvq_rows_f32 = ctypes.cast(self.cpu, P).value
        self.t.mvq_rows_cpu = self.t.mvq_rows_f32

    def _cpu(self, b, e, p):
        self.cpu_calls += 1
        a = ctypes.cast(p, ctypes.POINTER(MvqArg)).contents
        W, ws, x, out, y = self.mats[a.W]
        full = self.oracle.mvq_rows(W, ws, x, out, a.in_, a.group, a.bits, a.rowbytes)
        y[b:e] = full[b:e]

    def arg(self, W, ws, x, out, inn, group, bits, rowbytes):
        y = np.full(out, np.nan, np.float32)
        a = MvqArg(y.ctypes.data, W.ctypes.data, ws.ctypes.data, None, x.ctypes.data, inn,
                   (inn + group - 1) // group, group, bits, rowbytes)
        self.mats[W.ctypes.data] = (W, ws, x, out, y)
        return a, y

    def slot(self):
        return SLOT(self.t.mvq_rows_f32)


def _q(rng, out, inn, group, bits):
    rowbytes = (inn + group - 1) // group * group * bits // 8
    W = rng.integers(0, 256, out * rowbytes, dtype=np.uint8)
    ws = rng.uniform(0.001, 0.02, out * ((inn + group - 1) // group)).astype(np.float16)
    return W, ws.view(np.uint16), rng.standard_normal(inn).astype(np.float32), rowbytes


@pytest.fixture(scope="module")
def engine(cuda, oracle):
    from warp_b200 import ffi
    lib = ffi.load()
    eng = Engine(oracle)
    assert lib.waste_register_cuda(ctypes.byref(eng.t)) == b"CUDA sm_100a"
    _KEEP.append(eng)
    return eng


def test_register_fills_the_table(engine):
    from warp_b200 import ffi
    t = engine.t
    cpu = ctypes.cast(engine.cpu, P).value
    assert t.on_device == 1
    assert t.device_min_bytes == 256 << 10
    assert t.mvq_rows_f32 not in (None, cpu)
    assert t.mvq_rows_cpu == cpu
    for f in ("kda_step", "lutb_range", "vq_rows_p6", "vq_rows_e"):
        assert getattr(t, f) is None
    slot = t.mvq_rows_f32
    # idempotent: a second registration keeps the slot and the CPU snapshot
    assert ffi.load().waste_register_cuda(ctypes.byref(t)) == b"CUDA sm_100a"
    assert t.mvq_rows_f32 == slot and t.mvq_rows_cpu == cpu


@pytest.mark.parametrize("bits,group", [(4, 32), (8, 2304)])
def test_slot_runs_on_the_device(engine, oracle, bits, group):
    from warp_b200 import ffi
    lib = ffi.load()
    rng = np.random.default_rng(bits)
    out, inn = 512, 2304
    W, ws, x, rowbytes = _q(rng, out, inn, group, bits)
    before, calls = lib.warp_cuda_fallback_count(), engine.cpu_calls
    a, y = engine.arg(W, ws, x, out, inn, group, bits, rowbytes)
    engine.slot()(0, out, ctypes.addressof(a))
    want = oracle.mvq_rows(W, ws, x, out, inn, group, bits, rowbytes)
    assert rel_l2(y, want) < TOL_KERNEL
    # a sub-range writes only its rows
    y[:] = np.nan
    engine.slot()(100, 300, ctypes.addressof(a))
    assert rel_l2(y[100:300], want[100:300]) < TOL_KERNEL
    assert np.isnan(y[:100]).all() and np.isnan(y[300:]).all()
    assert lib.warp_cuda_fallback_count() == before
    assert engine.cpu_calls == calls


def test_slot_hands_unsupported_shapes_to_the_cpu(engine, oracle):
    from warp_b200 import ffi
    lib = ffi.load()
    rng = np.random.default_rng(5)
    out, inn, group, bits = 64, 240, 48, 4          # group not a multiple of 32
    W, ws, x, rowbytes = _q(rng, out, inn, group, bits)
    before, calls = lib.warp_cuda_fallback_count(), engine.cpu_calls
    a, y = engine.arg(W, ws, x, out, inn, group, bits, rowbytes)
    engine.slot()(0, out, ctypes.addressof(a))
    assert lib.warp_cuda_fallback_count() == before + 1
    assert engine.cpu_calls == calls + 1
    want = oracle.mvq_rows(W, ws, x, out, inn, group, bits, rowbytes)
    np.testing.assert_array_equal(y.view(np.uint32), want.view(np.uint32))


def _jobs(rec, lut_gu, lut_d, hidden, inter, ys):
    from warp_b200 import ffi
    h = C.parse_header(rec)
    nv_h, nv_i = hidden // 8, inter // 8
    J = (ffi.VqJob * 3)()
    specs = ((h["gate_off"], h["chan_corr_off"], lut_gu, 0, inter, nv_h),
             (h["up_off"], h["chan_corr_off"] + 2 * inter, lut_gu, nv_h * 3 * 256, inter, nv_h),
             (h["down_off"], h["chan_corr_off"] + 4 * inter, lut_d, 0, hidden, nv_i))
    for j, (io, so, lut, lo, m, nv) in enumerate(specs):
        J[j] = ffi.VqJob(ys[j].ctypes.data, rec.ctypes.data, rec.size, io, so, lut.ctypes.data,
                         lut.nbytes, lo, m, nv, 3, 256)
    return J


def test_vq3r_batch_matches_vq_rows(engine, oracle):
    """gate and up read two tables of one buffer (lut_off), down its own; the
    device results equal vq_rows bit for bit."""
    from warp_b200 import ffi
    lib = ffi.load()
    rng = np.random.default_rng(9)
    hidden, inter = 2304, 1024
    blocks = [rng.integers(0, 256, C.index_bytes(M, N), dtype=np.uint8)
              for M, N in ((inter, hidden), (inter, hidden), (hidden, inter))]
    scales = [rng.uniform(0.01, 0.05, n).astype(np.float16).view(np.uint16)
              for n in (inter, inter, hidden)]
    rec = np.frombuffer(C.write_record(2, 7, 9, blocks, scales, hidden, inter), np.uint8).copy()
    lut_gu = rng.standard_normal((2, hidden // 8, 3, 256)).astype(np.float32)
    lut_d = rng.standard_normal((inter // 8, 3, 256)).astype(np.float32)
    ys = [np.full(inter, np.nan, np.float32), np.full(inter, np.nan, np.float32),
          np.full(hidden, np.nan, np.float32)]
    J = _jobs(rec, lut_gu, lut_d, hidden, inter, ys)
    assert lib.waste_cuda_vq3r(J, 3) == 0
    wants = [oracle.vq_rows(blocks[0], scales[0], lut_gu[0], inter),
             oracle.vq_rows(blocks[1], scales[1], lut_gu[1], inter),
             oracle.vq_rows(blocks[2], scales[2], lut_d, hidden)]
    for y, want in zip(ys, wants):
        np.testing.assert_array_equal(y.view(np.uint32), want.view(np.uint32))
    # a job the device does not take: non-zero and nothing written
    for y in ys:
        y[:] = np.nan
    J[2].stages = 4
    assert lib.waste_cuda_vq3r(J, 3) != 0
    assert all(np.isnan(y).all() for y in ys)
    # after the release hook the mirrors are rebuilt on demand
    lib.waste_cuda_release_host_buffers()
    J[2].stages = 3
    assert lib.waste_cuda_vq3r(J, 3) == 0
    for y, want in zip(ys, wants):
        np.testing.assert_array_equal(y.view(np.uint32), want.view(np.uint32))


def test_vq3r_rejects_jobs_outside_their_buffers(engine):
    """Index, scale or table ranges past the buffers a job names are refused
    on the host, before anything is copied or launched."""
    from warp_b200 import ffi
    lib = ffi.load()
    rng = np.random.default_rng(10)
    hidden, inter = 256, 128
    blocks = [rng.integers(0, 256, C.index_bytes(M, N), dtype=np.uint8)
              for M, N in ((inter, hidden), (inter, hidden), (hidden, inter))]
    scales = [rng.uniform(0.01, 0.05, n).astype(np.float16).view(np.uint16)
              for n in (inter, inter, hidden)]
    rec = np.frombuffer(C.write_record(0, 1, 0, blocks, scales, hidden, inter), np.uint8).copy()
    lut_gu = rng.standard_normal((2, hidden // 8, 3, 256)).astype(np.float32)
    lut_d = rng.standard_normal((inter // 8, 3, 256)).astype(np.float32)
    ys = [np.full(inter, np.nan, np.float32), np.full(inter, np.nan, np.float32),
          np.full(hidden, np.nan, np.float32)]
    for field, value in (("lut_off", hidden // 8 * 3 * 256 + 1), ("sc_off", rec.size - 2),
                         ("idx_off", rec.size - 16), ("m", 10 ** 6)):
        J = _jobs(rec, lut_gu, lut_d, hidden, inter, ys)
        setattr(J[1], field, value)
        assert lib.waste_cuda_vq3r(J, 3) != 0, field
        assert all(np.isnan(y).all() for y in ys)
    J = _jobs(rec, lut_gu, lut_d, hidden, inter, ys)
    J[0].sc_off += 1                                   # odd: fp16 loads would misalign
    assert lib.waste_cuda_vq3r(J, 3) != 0
    assert all(np.isnan(y).all() for y in ys)
