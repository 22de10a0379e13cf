"""TEST INFRASTRUCTURE: ctypes bindings of the CPU oracle.

Two libraries, both built by oracle/Makefile:

* ``liboracle.so`` — warp_oracle.c, the restatement of the reference's
  expert-FFN arithmetic (the checker every GPU parity test uses);
* ``_ref/libwasteref.so`` — the reference engine's own C sources plus
  ref_shim.c, present only where the reference tree was available to compile
  (this is what pins the restatement; see tests/test_oracle_vs_ref.py).

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline import this
module.  The product (warp_b200/) never does.
"""
import ctypes
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libwasteref.so")
# The reference checkout: $WARP_REFERENCE, else a "reference" directory beside
# the repository's own.
REF_SRC = os.environ.get("WARP_REFERENCE",
                         os.path.normpath(os.path.join(HERE, "..", "..", "reference")))

_lock = threading.Lock()
_route_lock = threading.Lock()        # the oracle's layer router is process state
_lib = None
_ref = None

P = ctypes.c_void_p
I = ctypes.c_int
L = ctypes.c_long
F = ctypes.c_float
SZ = ctypes.c_size_t


def build(ref=False):
    """Compile liboracle.so (and the reference library when asked and the
    reference sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if ref and os.path.isdir(os.path.join(REF_SRC, "src")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={REF_SRC}"], check=True)


def _p(a):
    return a.ctypes.data_as(P) if a is not None else None


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(
                    os.path.join(HERE, "warp_oracle.c")):
                build()
            l = ctypes.CDLL(LIB)
            l.wo_f16.restype = F
            l.wo_f16.argtypes = [ctypes.c_uint16]
            l.wo_f32_to_f16.restype = ctypes.c_uint16
            l.wo_f32_to_f16.argtypes = [F]
            l.wo_books_decode.argtypes = [P, I, P, P]
            l.wo_lut_build.argtypes = [P, P, P, I, I]
            l.wo_lut_build_muladd.argtypes = [P, P, P, I, I]
            l.wo_vq_rows.argtypes = [P, P, P, P, I, I]
            l.wo_vq_dequant.argtypes = [P, P, P, P, I, I, I]
            l.wo_mvq_rows.argtypes = [P, P, P, P, I, I, I, I, SZ]
            l.wo_deq_rows.argtypes = [P, P, P, I, I, I, I, SZ]
            l.wo_deq_matmul_f64.argtypes = [P, P, P, P, I, I, I, I, I, SZ]
            l.wo_quant_q.argtypes = [P, I, I, I, I, P, P]
            l.wo_vq_encode.argtypes = [P, L, P, I, P, I]
            l.wo_block_indices.argtypes = [P, I, I, I, P]
            l.wo_quantize_vq.argtypes = [P, I, I, P, P, P, I]
            l.wo_qwen_route.restype = I
            l.wo_qwen_route.argtypes = [P, I, I, I, P, P]
            l.wo_swiglu.argtypes = [P, P, I]
            l.wo_router_logits.argtypes = [P, I, I, P, I, P]
            l.wo_route_scored.restype = I
            l.wo_route_scored.argtypes = [P, I, I, I, P, I, F, P, P, P]
            l.wo_set_router.argtypes = [I, I, P, F]
            l.wo_lut_build_se.argtypes = [P, P, P, I, I, I, I]
            l.wo_vq_quant_lut.argtypes = [P, I, I, I, P, P]
            l.wo_vq_rows_p6.argtypes = [P, P, P, P, P, I, I]
            l.wo_moe_layer.restype = I
            l.wo_moe_layer.argtypes = [P, I, I, I, I, I, P, P, P,
                                       P, P, P, P, P, P, I, I, I, P, P, P, P, P]
            _lib = l
    return _lib


def ref_available():
    return os.path.exists(REF_LIB) or os.path.isdir(os.path.join(REF_SRC, "src"))


def ref(nthreads=1):
    """The reference engine's own kernels (built from its sources).  The
    pool size is fixed by the first call in the process (0 = every core)."""
    global _ref
    with _lock:
        if _ref is None:
            if not os.path.exists(REF_LIB):
                if not os.path.isdir(os.path.join(REF_SRC, "src")):
                    raise RuntimeError("reference library not built and sources absent")
                subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={REF_SRC}"],
                               check=True)
            r = ctypes.CDLL(REF_LIB)
            r.ref_init.restype = I
            r.ref_init.argtypes = [I]
            r.ref_backend_name.restype = ctypes.c_char_p
            r.ref_mvq_rows.argtypes = [P, P, P, P, I, I, I, I, SZ, I]
            r.ref_deq_rows.argtypes = [P, P, P, I, I, I, I, SZ]
            r.ref_books_from_f16.argtypes = [P, I, I, I, P, P]
            r.ref_lutb.argtypes = [P, P, P, I, I, I, I, I, I]
            r.ref_vq_rows.argtypes = [P, P, P, P, I, I, I, I]
            r.ref_qwen_route.restype = I
            r.ref_qwen_route.argtypes = [P, I, I, I, P, P]
            r.ref_swiglu.argtypes = [P, P, I]
            r.ref_router_scores.argtypes = [I, P, P, I]
            r.ref_vq_quant_lut.argtypes = [P, I, I, I, P, P]
            r.ref_vq_rows_p6.argtypes = [P, P, P, P, P, I, I, I]
            r.ref_moe_new.restype = P
            r.ref_moe_new.argtypes = [P, I, I, I, I]
            r.ref_moe_free.argtypes = [P]
            r.ref_moe_experts.argtypes = [P, P, P, P, P, P, I]
            r.ref_shared_expert.argtypes = [P, P, P, P, P, P, P, I, I, P, P]
            r.waste_vq_encode.argtypes = [P, I, P, I, I, I, P, I]
            r.ref_matvec_f32.argtypes = [P, P, P, I, I]
            r.ref_threads.restype = I
            r.ref_init(nthreads)
            _ref = r
    return _ref


# ---------------------------------------------------------------- wrappers --

def f16_to_f32(h):
    return np.frombuffer(np.asarray(h, np.uint16).tobytes(), np.float16).astype(np.float32)


def books_decode(books_f16):
    """[n_books][256][8] fp16 (as uint16) -> (books, booksT) fp32, decoded as
    the engine's loader does (subnormals flushed)."""
    h = np.ascontiguousarray(books_f16, np.uint16)
    nb = h.size // (256 * 8)
    books = np.empty((nb, 256, 8), np.float32)
    booksT = np.empty((nb, 8, 256), np.float32)
    lib().wo_books_decode(_p(h), nb, _p(books), _p(booksT))
    return books, booksT


def lut_build(booksT, x, cb_base, muladd=False):
    x = np.ascontiguousarray(x, np.float32)
    nv = x.size // 8
    lut = np.empty((nv, 3, 256), np.float32)
    fn = lib().wo_lut_build_muladd if muladd else lib().wo_lut_build
    fn(_p(lut), _p(np.ascontiguousarray(booksT, np.float32)), _p(x), nv, cb_base)
    return lut


def lut_build_se(booksT, x, cb_base, stages, entries):
    x = np.ascontiguousarray(x, np.float32)
    nv = x.size // 8
    lut = np.empty((nv, stages, entries), np.float32)
    lib().wo_lut_build_se(_p(lut), _p(np.ascontiguousarray(booksT, np.float32)), _p(x), nv,
                          cb_base, stages, entries)
    return lut


def vq_quant_lut(lut):
    """lut [nv][st][en] fp32 -> (int8 table, per-32-position scales)."""
    lut = np.ascontiguousarray(lut, np.float32)
    nv, st, en = lut.shape
    q = np.empty(lut.shape, np.int8)
    sc = np.empty((nv + 31) // 32, np.float32)
    lib().wo_vq_quant_lut(_p(lut), nv, st, en, _p(q), _p(sc))
    return q, sc


def vq_rows_p6(idx, scale, lut8, lscale, M):
    nv = lut8.shape[0]
    y = np.empty(M, np.float32)
    lib().wo_vq_rows_p6(_p(y), _p(np.ascontiguousarray(idx, np.uint8)),
                        _p(np.ascontiguousarray(scale, np.uint16)),
                        _p(np.ascontiguousarray(lut8, np.int8)),
                        _p(np.ascontiguousarray(lscale, np.float32)), M, nv)
    return y


def vq_rows(idx, scale, lut, M):
    nv = lut.shape[0]
    y = np.empty(M, np.float32)
    lib().wo_vq_rows(_p(y), _p(np.ascontiguousarray(idx, np.uint8)),
                     _p(np.ascontiguousarray(scale, np.uint16)),
                     _p(np.ascontiguousarray(lut, np.float32)), M, nv)
    return y


def vq_dequant(idx, scale, books, M, N, cb_base):
    W = np.empty((M, N), np.float32)
    lib().wo_vq_dequant(_p(W), _p(np.ascontiguousarray(idx, np.uint8)),
                        _p(np.ascontiguousarray(scale, np.uint16)),
                        _p(np.ascontiguousarray(books, np.float32)), M, N, cb_base)
    return W


def mvq_rows(W, ws, x, out, inn, group, bits, rowbytes):
    y = np.empty(out, np.float32)
    lib().wo_mvq_rows(_p(y), _p(np.ascontiguousarray(W)), _p(np.ascontiguousarray(ws, np.uint16)),
                      _p(np.ascontiguousarray(x, np.float32)), out, inn, group, bits, rowbytes)
    return y


def deq_rows(W, ws, rows, cols, group, bits, rowbytes):
    d = np.empty((rows, cols), np.float32)
    lib().wo_deq_rows(_p(d), _p(np.ascontiguousarray(W)), _p(np.ascontiguousarray(ws, np.uint16)),
                      rows, cols, group, bits, rowbytes)
    return d


def deq_matmul_f64(W, ws, X, out, inn, group, bits, rowbytes):
    X = np.ascontiguousarray(X, np.float32).reshape(-1, inn)
    Y = np.empty((X.shape[0], out), np.float64)
    lib().wo_deq_matmul_f64(_p(Y), _p(np.ascontiguousarray(W)),
                            _p(np.ascontiguousarray(ws, np.uint16)), _p(X),
                            X.shape[0], out, inn, group, bits, rowbytes)
    return Y


def quant_q(W, group, bits):
    """quantize_q4g / quantize_q8g (convert.py:893-925) -> (payload u8, scales u16)."""
    W = np.ascontiguousarray(W, np.float32)
    rows, N = W.shape
    q = np.zeros(rows * N * bits // 8, np.uint8)
    s = np.empty(rows * (N // group), np.uint16)
    lib().wo_quant_q(_p(W), rows, N, group, bits, _p(q), _p(s))
    return q, s


def vq_encode(X, books, nthreads=os.cpu_count() or 1):
    X = np.ascontiguousarray(X, np.float32).reshape(-1, 8)
    B = np.ascontiguousarray(books, np.float32)
    st = B.shape[0]
    out = np.empty((X.shape[0], st), np.uint8)
    lib().wo_vq_encode(_p(X), X.shape[0], _p(B), st, _p(out), nthreads)
    return out


def block_indices(codes, M, N, stages=3):
    codes = np.ascontiguousarray(codes, np.uint8)
    nb = (M + 63) // 64
    out = np.empty(nb * (N // 8) * 64 * stages, np.uint8)
    lib().wo_block_indices(_p(codes), M, N, stages, _p(out))
    return out


def quantize_vq(W, books, nthreads=os.cpu_count() or 1):
    W = np.ascontiguousarray(W, np.float32)
    M, N = W.shape
    codes = np.empty((M * N // 8, 3), np.uint8)
    scales = np.empty(M, np.uint16)
    lib().wo_quantize_vq(_p(W), M, N, _p(np.ascontiguousarray(books, np.float32)),
                         _p(codes), _p(scales), nthreads)
    return codes, scales


def qwen_route(logits, K, renorm):
    logits = np.ascontiguousarray(logits, np.float32)
    idx = np.empty(K, np.int32)
    w = np.empty(K, np.float32)
    rc = lib().wo_qwen_route(_p(logits), logits.size, K, int(renorm), _p(idx), _p(w))
    return rc, idx, w


def route_scored(logits, K, func, bias=None, renorm=True, routed_scale=1.0):
    """moe_layer's routing for one token -> (rc, idx, w, scores)."""
    logits = np.ascontiguousarray(logits, np.float32)
    E = logits.size
    idx = np.empty(K, np.int32)
    w = np.empty(K, np.float32)
    sc = np.empty(E, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    rc = lib().wo_route_scored(_p(logits), E, K, int(func), _p(b), int(renorm),
                               float(routed_scale), _p(idx), _p(w), _p(sc))
    return rc, idx, w, sc


def swiglu(g, u):
    g = np.array(g, np.float32, copy=True)
    lib().wo_swiglu(_p(g), _p(np.ascontiguousarray(u, np.float32)), g.size)
    return g


def router_logits(X, router):
    """Router logits of many tokens, X [T][hid] -> [T][E], summed as
    moe_layer sums them."""
    X = np.ascontiguousarray(X, np.float32)
    T, hid = X.shape
    R = np.ascontiguousarray(router, np.float32)
    E = R.shape[0]
    out = np.empty((T, E), np.float32)
    lib().wo_router_logits(_p(X), T, hid, _p(R), E, _p(out))
    return out


def moe_layer(x, hid, inter, E, K, renorm, router, recs, booksT, shared=None,
              shared_gate=None, route=None):
    """One MoE layer for one token.  recs: list of E numpy uint8 records.
    shared: dict(gate_w, gate_s, up_w, up_s, down_w, down_s, group, bits,
    inter) or None.  route: None for Qwen's router, or dict(func, bias,
    routed_scale) for moe_layer's."""
    bias = None
    if route is not None and route.get("bias") is not None:
        bias = np.ascontiguousarray(route["bias"], np.float32)
    lib()
    with _route_lock:
        if route is None:
            lib().wo_set_router(0, 0, None, 1.0)
        else:
            lib().wo_set_router(1, int(route["func"]), _p(bias),
                                float(route.get("routed_scale", 1.0)))
        try:
            return _moe_layer(x, hid, inter, E, K, renorm, router, recs, booksT, shared,
                              shared_gate)
        finally:
            lib().wo_set_router(0, 0, None, 1.0)


def _moe_layer(x, hid, inter, E, K, renorm, router, recs, booksT, shared, shared_gate):
    arr = (P * E)(*[r.ctypes.data for r in recs])
    out = np.empty(hid, np.float32)
    idx = np.empty(K, np.int32)
    w = np.empty(K, np.float32)
    acc = np.empty((K, hid), np.float32)
    s = shared or {}
    rc = lib().wo_moe_layer(
        _p(np.ascontiguousarray(x, np.float32)), hid, inter, E, K, int(renorm),
        _p(np.ascontiguousarray(router, np.float32)), ctypes.cast(arr, P),
        _p(np.ascontiguousarray(booksT, np.float32)),
        _p(s.get("gate_w")), _p(s.get("gate_s")), _p(s.get("up_w")), _p(s.get("up_s")),
        _p(s.get("down_w")), _p(s.get("down_s")), s.get("group", 32), s.get("bits", 4),
        s.get("inter", 0), _p(shared_gate), _p(out), _p(idx), _p(w), _p(acc))
    if rc != 0:
        raise ValueError("oracle moe_layer rejected its arguments")
    return out, idx, w, acc
