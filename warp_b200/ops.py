"""Torch-tensor front end of the C ABI (include/warp_cuda.h).

Names follow the reference functions whose arithmetic each call computes:

    mvq_matvec      waste_mvq_rows_f32      (src/model.c:423-519)
    vq_build_lut    vq_build_lut / lutb_range_avx512 (model.c:3864, simd_avx512.c:90)
    vq_apply        vq_apply / vq_rows      (model.c:4152, 3909-3977)
    vq_dequant      tools/kimi_ref.py:240-273 (expert dequant)
    vq4p_lut        vq_build_lut (4 x 64) + vq_quant_lut (model.c:3815, 4063)
    vq4p_apply      waste_vq_rows_p6        (model.c:4076-4113)
    vq_encode       waste_vq_encode         (src/vq.c:99)
    qwen_moe_route  waste_qwen_moe_route    (src/qwen_moe.c:10-44)
    MoELayer        qwen_moe_layer / moe_layer (model.c:8180, 5488)

Every tensor argument must already be on the CUDA device; calls are
asynchronous on torch's current stream.  A failure raises ffi.WarpError.
"""
import ctypes

import torch

from . import ffi
from .container import ENTRIES, STAGES, VEC, parse_header


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("warp_b200 ops take CUDA tensors")


def mvq_matvec(W, ws, X, out, in_, group, bits, rowbytes=None):
    """Y[b][o] = sum_k f16(ws[o,k]) * sum_i q(o,k*g+i) * X[b][k*g+i]."""
    _cuda(W, ws, X)
    if rowbytes is None:
        rowbytes = (in_ + group - 1) // group * group * bits // 8
    X2 = X.reshape(-1, in_).contiguous()
    if X2.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("activations must be fp32 or bf16")
    Y = torch.empty(X2.shape[0], out, dtype=torch.float32, device=X.device)
    ffi.check(ffi.load().warp_mvq_matvec(
        _p(W), _p(ws), _p(X2), int(X2.dtype == torch.bfloat16), _p(Y), X2.shape[0], out,
        in_, group, bits, rowbytes, _stream()))
    return Y


def vq_build_lut(booksT, x, cb_base):
    """lut[v][s][c] = FMA chain over d of x[8v+d] * booksT[cb_base+s][d][c]."""
    _cuda(booksT, x)
    nv = x.numel() // VEC
    lut = torch.empty(nv, STAGES, ENTRIES, dtype=torch.float32, device=x.device)
    ffi.check(ffi.load().warp_vq_lut_build(_p(lut), _p(booksT), _p(x.contiguous()), nv,
                                           cb_base, _stream()))
    return lut


def vq_apply(idx, scale, lut, M, ordered=False):
    """y[r] = f16(scale[r]) * sum_v T_v[i0] + T_v[i1] + T_v[i2]."""
    _cuda(idx, scale, lut)
    y = torch.empty(M, dtype=torch.float32, device=lut.device)
    ffi.check(ffi.load().warp_vq_apply(_p(y), _p(idx), _p(scale), _p(lut), M, lut.shape[0],
                                       int(ordered), _stream()))
    return y


def vq4p_lut(booksT, x, cb_base=0):
    """VQ4P int8 table of x: (q [nv][4][64] int8, lscale [ceil(nv/32)])."""
    _cuda(booksT, x)
    nv = x.numel() // VEC
    q = torch.empty(nv, 4, 64, dtype=torch.int8, device=x.device)
    ls = torch.empty((nv + 31) // 32, dtype=torch.float32, device=x.device)
    ffi.check(ffi.load().warp_vq4p_lut(_p(q), _p(ls), _p(booksT.contiguous()), booksT.shape[0],
                                       _p(x.contiguous()), nv, cb_base, _stream()))
    return q, ls


def vq4p_apply(idx, scale, q, lscale, M):
    """waste_vq_rows_p6: y[r] = f16(scale[r]) * sum_blk lscale[blk] * sum(lookups)."""
    _cuda(idx, scale, q, lscale)
    y = torch.empty(M, dtype=torch.float32, device=q.device)
    ffi.check(ffi.load().warp_vq4p_apply(_p(y), _p(idx), _p(scale), _p(q), _p(lscale), M,
                                         q.shape[0], _stream()))
    return y


def vq_matmul(X, idx, scale, books, M, cb_base=0):
    """Y[t][r] = f16(scale[r]) * sum_k W~[r][k] X[t][k] on the tensor cores
    (fp16 operands, fp32 accumulation); X [T][N] fp32 -> Y [T][M] fp32."""
    _cuda(X, idx, scale, books)
    X2 = X.reshape(-1, X.shape[-1]).contiguous().float()
    T, N = X2.shape
    Y = torch.empty(T, M, dtype=torch.float32, device=X.device)
    ffi.check(ffi.load().warp_vq_matmul(_p(Y), _p(X2), T, _p(idx), _p(scale), _p(books), M, N,
                                        cb_base, _stream()))
    return Y


def umma_status(clear=True):
    ffi.check(ffi.load().warp_umma_status(int(clear)))


def vq_dequant(idx, scale, books, M, N, cb_base):
    """Dequantized VQ3R matrix, fp32 [M][N], bit-exact."""
    _cuda(idx, scale, books)
    W = torch.empty(M, N, dtype=torch.float32, device=books.device)
    ffi.check(ffi.load().warp_vq_dequant(_p(W), _p(idx), _p(scale), _p(books), M, N,
                                         cb_base, _stream()))
    return W


def vq_encode(X, books):
    """Residual nearest-centroid codes, X [n][8] fp32, books [stages][256][8]."""
    _cuda(X, books)
    X = X.reshape(-1, VEC).contiguous()
    codes = torch.empty(X.shape[0], books.shape[0], dtype=torch.uint8, device=X.device)
    ffi.check(ffi.load().warp_vq_encode(_p(X), X.shape[0], _p(books.contiguous()),
                                        books.shape[0], _p(codes), _stream()))
    return codes


def qwen_moe_route(logits, K, renorm=True):
    """Softmax top-k in selection order; logits [T][E]."""
    _cuda(logits)
    L = logits.reshape(-1, logits.shape[-1]).contiguous().float()
    T, E = L.shape
    idx = torch.empty(T, K, dtype=torch.int32, device=L.device)
    w = torch.empty(T, K, dtype=torch.float32, device=L.device)
    ffi.check(ffi.load().warp_qwen_route(_p(L), T, E, K, int(renorm), _p(idx), _p(w),
                                         _stream()))
    return idx, w


def moe_route(logits, K, score_func, bias=None, renorm=True, routed_scale=1.0):
    """moe_layer's routing (router_scores + biased selection + renorm +
    routed_scale); logits [T][E]."""
    _cuda(logits, bias)
    L = logits.reshape(-1, logits.shape[-1]).contiguous().float()
    T, E = L.shape
    idx = torch.empty(T, K, dtype=torch.int32, device=L.device)
    w = torch.empty(T, K, dtype=torch.float32, device=L.device)
    ffi.check(ffi.load().warp_moe_route(_p(L), T, E, K, int(score_func), _p(bias), int(renorm),
                                        float(routed_scale), _p(idx), _p(w), _stream()))
    return idx, w


def rmsnorm(x, w=None, eps=1e-6, out=None):
    """waste_rmsnorm over the last dimension."""
    _cuda(x, w)
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    if out is None:
        out = torch.empty_like(x2)
    ffi.check(ffi.load().warp_rmsnorm(_p(x2), _p(w), _p(out), x2.shape[0], x2.shape[1],
                                      eps, _stream()))
    return out


class MoELayer:
    """One resident MoE layer on the device (warp_moe_layer_*).

    bank: uint8 CUDA tensor of E expert records (rec_bytes each, sorted by id);
    books/booksT: the layer's decoded codebooks; router: fp32 [E][hidden];
    shared: optional dict(gate_w, gate_s, up_w, up_s, down_w, down_s, inter,
    group, bits) of CUDA tensors; shared_gate: optional fp32 [hidden].
    tile_bank (default) re-tiles the bank in place on creation (see
    warp_moe_desc.tile_bank): read the records you need in container layout
    before creating the layer.
    """

    def __init__(self, bank, rec_bytes, books, booksT, router, hidden, inter, n_experts,
                 top_k, renorm=True, shared=None, shared_gate=None, max_tokens=1,
                 tile_bank=True, ep_rank=0, ep_size=1, prefill_tokens=0, router_kind=0,
                 score_func=0, score_bias=None, routed_scale=1.0, ep_mode=0):
        _cuda(bank, books, booksT, router, score_bias)
        self.keep = [bank, books, booksT, router, shared_gate, score_bias] + \
            (list(shared.values()) if shared else [])
        self.hidden, self.inter, self.E, self.K = hidden, inter, n_experts, top_k
        self.max_tokens = max_tokens
        d = ffi.MoEDesc()
        d.hidden, d.inter, d.n_experts, d.top_k, d.renorm = hidden, inter, n_experts, top_k, int(renorm)
        d.bank, d.rec_bytes = bank.data_ptr(), rec_bytes
        d.booksT, d.books, d.n_books = booksT.data_ptr(), books.data_ptr(), books.shape[0]
        d.router = router.data_ptr()
        if shared:
            d.shared_gate_w = shared["gate_w"].data_ptr()
            d.shared_up_w = shared["up_w"].data_ptr()
            d.shared_down_w = shared["down_w"].data_ptr()
            d.shared_gate_s = shared["gate_s"].data_ptr()
            d.shared_up_s = shared["up_s"].data_ptr()
            d.shared_down_s = shared["down_s"].data_ptr()
            d.shared_inter, d.shared_group = shared["inter"], shared["group"]
            d.shared_bits = shared["bits"]
        if shared_gate is not None:
            d.shared_gate = shared_gate.data_ptr()
        d.tile_bank = int(tile_bank)
        d.ep_rank, d.ep_size = int(ep_rank), int(ep_size)
        d.prefill_tokens = int(prefill_tokens)
        d.router_kind, d.score_func = int(router_kind), int(score_func)
        if score_bias is not None:
            d.score_bias = score_bias.data_ptr()
        d.routed_scale = float(routed_scale)
        d.ep_mode = int(ep_mode)
        self.ep_rank, self.ep_size = int(ep_rank), int(ep_size)
        self.desc = d
        h = ctypes.c_void_p()
        ffi.check(ffi.load().warp_moe_layer_create(ctypes.byref(d), max_tokens,
                                                   ctypes.byref(h)))
        self.handle = h

    def forward(self, x, residual=None, out=None, want_route=False):
        _cuda(x)
        x2 = x.reshape(-1, self.hidden)
        T = x2.shape[0]
        if out is None:
            out = torch.empty(T, self.hidden, dtype=torch.float32, device=x.device)
        idx = w = None
        if want_route:
            idx = torch.empty(T, self.K, dtype=torch.int32, device=x.device)
            w = torch.empty(T, self.K, dtype=torch.float32, device=x.device)
        ffi.check(ffi.load().warp_moe_layer_forward(
            self.handle, _p(x2), T, _p(residual), _p(out), _p(idx), _p(w), _stream()))
        return (out, idx, w) if want_route else out

    def forward_block(self, h, out, norm_w=None, eps=1e-6, want_route=False):
        """out = h + MoE(RMSNorm(h) * norm_w): the norm kernel into the
        layer's buffer, then the layer with residual h (warp_moe_block_forward);
        out must not alias h."""
        _cuda(h, out, norm_w)
        h2 = h.reshape(-1, self.hidden)
        T = h2.shape[0]
        idx = w = None
        if want_route:
            idx = torch.empty(T, self.K, dtype=torch.int32, device=h.device)
            w = torch.empty(T, self.K, dtype=torch.float32, device=h.device)
        ffi.check(ffi.load().warp_moe_block_forward(
            self.handle, _p(h2), T, _p(norm_w), float(eps), _p(out), _p(idx), _p(w), _stream()))
        return (out, idx, w) if want_route else out

    def prefill(self, x, residual=None, out=None, want_route=False):
        """The layer for T tokens on the tensor cores (warp_moe_layer_prefill)."""
        _cuda(x)
        x2 = x.reshape(-1, self.hidden).contiguous()
        T = x2.shape[0]
        if out is None:
            out = torch.empty(T, self.hidden, dtype=torch.float32, device=x.device)
        idx = w = None
        if want_route:
            idx = torch.empty(T, self.K, dtype=torch.int32, device=x.device)
            w = torch.empty(T, self.K, dtype=torch.float32, device=x.device)
        ffi.check(ffi.load().warp_moe_layer_prefill(
            self.handle, _p(x2), T, _p(residual), _p(out), _p(idx), _p(w), _stream()))
        return (out, idx, w) if want_route else out

    def slots_per_token(self):
        """S: top_k route slots plus the shared expert's column blocks."""
        return ffi.load().warp_moe_layer_slots_per_token(self.handle)

    def slots(self, T=1, device=None):
        """A zeroed slot buffer for forward_ep: [T][S][hidden] fp32."""
        return torch.zeros(T, self.slots_per_token(), self.hidden, dtype=torch.float32,
                           device=device)

    def forward_ep(self, x, slots, want_route=False):
        """Expert-parallel first half: this rank's routed outputs and its
        share of the shared expert into slots (warp_moe_layer_forward_ep)."""
        _cuda(x, slots)
        x2 = x.reshape(-1, self.hidden)
        T = x2.shape[0]
        if slots.shape != (T, self.slots_per_token(), self.hidden) or not slots.is_contiguous():
            raise ValueError("slots must be a contiguous [T][S][hidden] tensor (S: "
                             "slots_per_token)")
        idx = w = None
        if want_route:
            idx = torch.empty(T, self.K, dtype=torch.int32, device=x.device)
            w = torch.empty(T, self.K, dtype=torch.float32, device=x.device)
        ffi.check(ffi.load().warp_moe_layer_forward_ep(
            self.handle, _p(x2), T, _p(slots), _p(idx), _p(w), _stream()))
        return (idx, w) if want_route else None

    def combine(self, slots, residual=None, out=None):
        """Second half, after the slots were all-reduced over the ranks."""
        _cuda(slots)
        T = slots.shape[0]
        if out is None:
            out = torch.empty(T, self.hidden, dtype=torch.float32, device=slots.device)
        ffi.check(ffi.load().warp_moe_layer_combine(self.handle, _p(slots), T, _p(residual),
                                                    _p(out), _stream()))
        return out

    PHASES = ("router", "gate_up_gather", "swiglu", "down_gather", "shared", "combine")

    def set_timing(self, on):
        ffi.check(ffi.load().warp_moe_layer_set_timing(self.handle, int(on)))

    def collect(self):
        """Add the phase times of the last graph replay (timing on at capture)."""
        ffi.check(ffi.load().warp_moe_layer_collect(self.handle))

    def timings(self):
        """(forwards, {phase: total ms}) since set_timing(True)."""
        ms = (ctypes.c_double * 6)()
        n = ffi.load().warp_moe_layer_timings(self.handle, ms)
        return n, dict(zip(self.PHASES, list(ms)))

    def status(self):
        ffi.check(ffi.load().warp_moe_layer_status(self.handle, _stream()))

    def close(self):
        if getattr(self, "handle", None):
            ffi.load().warp_moe_layer_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def record_offsets(bank_bytes_first_record):
    return parse_header(bank_bytes_first_record)
