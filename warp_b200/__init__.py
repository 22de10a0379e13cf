"""warp_b200 — B200 (sm_100a) backend for WARP's quantized expert FFN.

The compute lives in libwarp_cuda.so (warp_b200/csrc, C ABI in
include/warp_cuda.h).  This package is its host side: the ctypes binding
(ffi), torch-tensor entry points named after the reference functions (ops),
the container layout (container) and seeded synthetic experts (synth).
"""
__version__ = "0.1"


def lib():
    """The loaded libwarp_cuda.so; raises if it was not built."""
    from . import ffi
    return ffi.load()
