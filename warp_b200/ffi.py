"""ctypes binding of libwarp_cuda.so (include/warp_cuda.h).

The library is built in-tree by ``python -m warp_b200.build``.  Loading it
never falls back to anything: a missing or unloadable library raises.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libwarp_cuda.so")

P = ctypes.c_void_p
I = ctypes.c_int
I64 = ctypes.c_int64
SZ = ctypes.c_size_t
F = ctypes.c_float

# every function include/warp_cuda.h declares: name -> (restype, argtypes)
SIGNATURES = {
    "warp_version": (ctypes.c_char_p, []),
    "warp_last_error": (ctypes.c_char_p, []),
    "warp_device_ok": (I, [I]),
    "warp_launch_count": (ctypes.c_uint64, []),
    "waste_register_cuda": (ctypes.c_char_p, [P]),
    "waste_cuda_vq3r": (I, [P, I]),
    "waste_cuda_release_host_buffers": (None, []),
    "warp_cuda_fallback_count": (ctypes.c_ulonglong, []),
    "warp_cuda_stats": (I, [P]),
    "waste_metal_vq3r": (I, [P, I]),
    "waste_register_metal": (ctypes.c_char_p, [P]),
    "waste_metal_release_host_buffers": (None, []),
    "waste_metal_selftest": (None, []),
    "warp_mvq_matvec": (I, [P, P, P, I, P, I, I, I, I, I, SZ, P]),
    "warp_mvq_status": (I, [I]),
    "warp_vq_lut_build": (I, [P, P, P, I, I, P]),
    "warp_vq_apply": (I, [P, P, P, P, I, I, I, P]),
    "warp_vq_apply_noalloc": (I, [P, P, P, P, I, I, P]),
    "warp_vq_dequant": (I, [P, P, P, P, I, I, I, P]),
    "warp_vq4p_lut": (I, [P, P, P, I, P, I, I, P]),
    "warp_vq4p_apply": (I, [P, P, P, P, P, I, I, P]),
    "warp_vq_matmul": (I, [P, P, I, P, P, P, I, I, I, P]),
    "warp_umma_status": (I, [I]),
    "warp_vq_encode": (I, [P, I64, P, I, P, P]),
    "warp_qwen_route": (I, [P, I, I, I, I, P, P, P]),
    "warp_moe_route": (I, [P, I, I, I, I, P, I, F, P, P, P]),
    "warp_rmsnorm": (I, [P, P, P, I, I, F, P]),
    "warp_moe_layer_create": (I, [P, I, P]),
    "warp_moe_layer_destroy": (None, [P]),
    "warp_moe_layer_status": (I, [P, P]),
    "warp_moe_layer_forward": (I, [P, P, I, P, P, P, P, P]),
    "warp_moe_block_forward": (I, [P, P, I, P, F, P, P, P, P]),
    "warp_moe_layer_forward_ep": (I, [P, P, I, P, P, P, P]),
    "warp_moe_layer_combine": (I, [P, P, I, P, P, P]),
    "warp_moe_layer_slots_per_token": (I, [P]),
    "warp_moe_layer_prefill": (I, [P, P, I, P, P, P, P, P]),
    "warp_moe_layer_set_timing": (I, [P, I]),
    "warp_moe_layer_timings": (I, [P, P]),
    "warp_moe_layer_collect": (I, [P]),
}


class WarpError(RuntimeError):
    """A warp_status other than WARP_OK, with warp_last_error()'s text."""

    def __init__(self, rc, msg):
        super().__init__(f"warp_b200 error {rc}: {msg}")
        self.rc = rc


class MoEDesc(ctypes.Structure):
    """warp_moe_desc (include/warp_cuda.h)."""
    _fields_ = [
        ("hidden", I), ("inter", I), ("n_experts", I), ("top_k", I), ("renorm", I),
        ("bank", P), ("rec_bytes", SZ), ("booksT", P), ("books", P), ("n_books", I),
        ("router", P),
        ("shared_gate_w", P), ("shared_up_w", P), ("shared_down_w", P),
        ("shared_gate_s", P), ("shared_up_s", P), ("shared_down_s", P),
        ("shared_inter", I), ("shared_group", I), ("shared_bits", I),
        ("shared_gate", P), ("tile_bank", I), ("ep_rank", I), ("ep_size", I),
        ("prefill_tokens", I), ("router_kind", I), ("score_func", I), ("score_bias", P),
        ("routed_scale", F), ("ep_mode", I),
    ]


class VqJob(ctypes.Structure):
    """warp_vq_job == waste_vq_job (waste_metal.h:31-40)."""
    _fields_ = [
        ("y", P), ("rec", P), ("rec_bytes", SZ), ("idx_off", ctypes.c_uint32),
        ("sc_off", ctypes.c_uint32), ("lut", P), ("lut_bytes", SZ),
        ("lut_off", ctypes.c_uint32), ("m", I), ("nv", I), ("stages", I), ("entries", I),
    ]


_lib = None


def load():
    """The loaded library; raises if it is absent or does not load."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m warp_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc):
    if rc != 0:
        raise WarpError(rc, load().warp_last_error().decode(errors="replace"))
    return rc
