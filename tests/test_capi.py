"""The C-ABI library builds, loads without a GPU and exports every function
include/*.h declares; the Python binding covers exactly those."""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        for m in re.finditer(r"WARP_API\s+[\w\s\*]+?\b(\w+)\s*\(", src):
            names.add(m.group(1))
    return names


@pytest.fixture(scope="module")
def lib():
    from warp_b200 import build, ffi
    build.build()
    return ffi.load()


def test_exports_every_declared_symbol(lib):
    declared = _declared()
    assert len(declared) >= 15
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_matches_header(lib):
    from warp_b200 import ffi
    assert set(ffi.SIGNATURES) == _declared()


def test_loads_without_device(lib):
    assert lib.warp_version().startswith(b"warp_b200")
    # no CUDA device in the build container: the library reports that
    # instead of failing to load or crashing
    import torch
    if not torch.cuda.is_available():
        assert lib.warp_device_ok(0) == 0
        assert lib.waste_register_cuda(ctypes.c_void_p(0)) is None


def test_argument_errors_are_returned(lib):
    from warp_b200 import ffi
    rc = lib.warp_mvq_matvec(None, None, None, 0, None, 1, 1, 32, 32, 4, 16, None)
    assert rc == -1
    assert b"NULL" in lib.warp_last_error()
    rc = lib.warp_moe_layer_create(None, 1, None)
    assert rc == -1
