"""Failure paths made on the host, none of which faults the device:

* a bank whose record header is corrupted (magic, expert id, offsets) into
  warp_moe_layer_create: WARP_E_FORMAT with the record named, nothing
  allocated, and the context stays usable (a good layer runs afterwards);
* WARP_CUDA_DISABLE=1: waste_register_cuda declines (NULL) on a machine with
  a device and leaves the engine's table as it found it, so the engine keeps
  its CPU kernels (backend.c:108-125 treats NULL as "no accelerator").
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from warp_b200 import container as C

pytestmark = pytest.mark.gpu

H, INTER, E, K = 256, 128, 8, 2
WARP_E_FORMAT = -6


def _layer(cuda, seed=5):
    from warp_b200 import synth
    bank = synth.random_bank(E, H, INTER, seed, device=cuda)
    router = synth.router_matrix(E, H, seed + 1, device=cuda)
    return synth.SyntheticLayer(bank, router)


# the fields of the WEXP header (waste_format.h:98-130), in C.HDR's order
FIELD = dict(magic=0, layer=1, expert_id=2, fmt=3, flags=4, codebook_id=5, gate_off=9,
             up_off=10, down_off=11, chan_corr_off=12)


def _corrupt(layer, recs, field, value):
    """Overwrite one header field of the records `recs` in the device bank."""
    rb = layer.bank.rec_bytes
    for rec in recs:
        raw = layer.bank.bank[rec * rb:rec * rb + C.HDR.size].cpu().numpy().tobytes()
        f = list(C.HDR.unpack(raw))
        f[FIELD[field]] = value
        layer.bank.bank[rec * rb:rec * rb + C.HDR.size] = torch.from_numpy(
            np.frombuffer(C.HDR.pack(*f), np.uint8).copy()).to(layer.bank.bank.device)


@pytest.mark.parametrize("field,value,recs,says", [
    ("magic", 0x12345678, [3], "record 3 is not"),
    ("expert_id", 6, [5], "record 5 is not"),
    ("fmt", 3, [2], "record 2 is not"),
    ("codebook_id", 7, [1], "record 1 is not"),
    ("down_off", 16, list(range(E)), "offsets do not fit"),     # consistent but impossible
    ("codebook_id", 200, list(range(E)), "offsets do not fit"), # books past the table
])
def test_corrupted_header_is_a_format_error(cuda, field, value, recs, says):
    from warp_b200 import ffi
    lay = _layer(cuda)
    _corrupt(lay, recs, field, value)
    before = lay.bank.bank.clone()
    with pytest.raises(ffi.WarpError) as ei:
        lay.moe(K, tile_bank=True)
    assert ei.value.rc == WARP_E_FORMAT, ei.value
    assert says in str(ei.value), str(ei.value)
    # the refusal comes before any re-tiling: the bank is untouched
    torch.cuda.synchronize()
    assert torch.equal(lay.bank.bank, before)
    # the context is still good: a clean layer builds and runs
    good = _layer(cuda, seed=9)
    m = good.moe(K)
    try:
        x = torch.randn(1, H, device=cuda)
        out = m.forward(x)
        m.status()
        assert torch.isfinite(out).all()
    finally:
        m.close()


def test_disable_declines_registration(cuda, monkeypatch):
    from warp_b200 import ffi
    from test_gpu_boundary import Kernels, SLOT, P
    lib = ffi.load()
    fake = SLOT(lambda b, e, p: None)
    t = Kernels()
    t.mvq_rows_f32 = ctypes.cast(fake, P).value
    t.mvq_rows_cpu = t.mvq_rows_f32
    snap = bytes(t)
    monkeypatch.setenv("WARP_CUDA_DISABLE", "1")
    assert lib.waste_register_cuda(ctypes.byref(t)) is None
    assert bytes(t) == snap, "a declined registration must leave the table alone"
    # "0" is not a request to decline
    monkeypatch.setenv("WARP_CUDA_DISABLE", "0")
    assert lib.waste_register_cuda(ctypes.byref(t)) == b"CUDA sm_100a"
    assert t.on_device == 1 and t.mvq_rows_cpu == ctypes.cast(fake, P).value
    assert os.environ["WARP_CUDA_DISABLE"] == "0"
