"""The drop-in at engine level: the reference's own engine and its
tests/test_forward.c, every source unchanged, built by oracle/Makefile
(`make engine`) with -DWASTE_ENABLE_CUDA=1 -DWASTE_ENABLE_METAL=1 and linked
against libwarp_cuda.so, which answers waste_register_cuda and the three
Metal hooks.  The container is the reference's seed-0 test container
(tests/golden/kimi_tiny.waste, written by tools/make_test_container.py).

The engine compares against itself, as tests/run.sh does (run.sh:787-800):
  * WASTE_METAL_MOE=1 sends every MoE layer's routed-expert applies through
    waste_metal_vq3r, here the CUDA batch apply.  Against the same SIMD
    build with the device declined (WARP_CUDA_DISABLE=1), the logits must be
    bit-identical: the device apply is bit-exact to vq_rows.
  * Against WASTE_BACKEND=cpu (the portable kernels), run.sh's logit rule:
    the same argmax and every logit within 1e-3.
  * WARP_CUDA_DEVICE_MIN_KB=0 also sends every trunk matvec through run_rows
    to the device slot; the same rule against the CPU backend.
WARP_CUDA_STATS makes the library report, at the engine's exit, how many
slot calls and batch applies the device ran, so a run that quietly stayed on
the CPU fails.
"""
import json
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENGINE = os.path.join(ROOT, "oracle", "_ref", "engine", "test_forward")
CONTAINER = os.path.join(ROOT, "tests", "golden", "kimi_tiny.waste")
IDS = ",".join(str(i) for i in (1, 17, 33, 49, 65, 81, 97, 113, 129, 145, 161, 177, 193, 209,
                                225, 241))
LOGIT_EPS = 1e-3          # tests/run.sh:120


def _run(tmp_path, name, env):
    if not os.path.exists(ENGINE):
        pytest.skip("engine not built (oracle/Makefile `make engine` needs the reference)")
    out = str(tmp_path / f"{name}.bin")
    stats = str(tmp_path / f"{name}.stats")
    e = dict(os.environ)
    for k in ("WASTE_BACKEND", "WASTE_METAL_MOE", "WARP_CUDA_DISABLE",
              "WARP_CUDA_DEVICE_MIN_KB", "WARP_CUDA_STATS"):
        e.pop(k, None)
    e.update(env)
    e["WARP_CUDA_STATS"] = stats
    r = subprocess.run([ENGINE, CONTAINER, IDS, out, "0"], env=e, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    logits = np.fromfile(out, np.float32)
    assert logits.size == 256 and np.isfinite(logits).all()
    st = None
    if os.path.exists(stats):
        with open(stats) as f:
            st = json.loads(f.read().strip().splitlines()[-1])
    return logits, st, r.stdout + r.stderr


def _logitcmp(a, b):
    assert int(np.argmax(a)) == int(np.argmax(b))
    assert float(np.abs(a - b).max()) < LOGIT_EPS


def test_engine_runs_with_the_library_and_no_device(tmp_path):
    """CPU only: the engine linked against the library runs; with the device
    declined the Metal hook answers non-zero and the engine's own loop does
    the work, so the logits equal the plain SIMD run's."""
    base, _, out = _run(tmp_path, "simd", {"WARP_CUDA_DISABLE": "1", "WASTE_CACHE_MB": "8"})
    assert "backend CUDA" not in out
    hook, st, _ = _run(tmp_path, "hook", {"WARP_CUDA_DISABLE": "1", "WASTE_CACHE_MB": "8",
                                          "WASTE_METAL_MOE": "1"})
    assert np.array_equal(base.view(np.uint32), hook.view(np.uint32))


@pytest.mark.gpu
def test_engine_moe_hook_on_the_device(cuda, tmp_path):
    simd, _, _ = _run(tmp_path, "simd", {"WARP_CUDA_DISABLE": "1", "WASTE_CACHE_MB": "8"})
    cpu, _, _ = _run(tmp_path, "cpu", {"WASTE_BACKEND": "cpu", "WASTE_CACHE_MB": "8"})
    dev, st, out = _run(tmp_path, "dev", {"WASTE_METAL_MOE": "1", "WASTE_CACHE_MB": "8"})
    assert "backend CUDA sm_100a" in out, out
    assert st is not None and st["vq3r_calls"] > 0 and st["vq3r_jobs"] > 0, st
    # the device apply is vq_rows bit for bit
    assert np.array_equal(dev.view(np.uint32), simd.view(np.uint32))
    _logitcmp(dev, cpu)


@pytest.mark.gpu
def test_engine_trunk_matvec_on_the_device(cuda, tmp_path):
    cpu, _, _ = _run(tmp_path, "cpu", {"WASTE_BACKEND": "cpu", "WASTE_CACHE_MB": "8"})
    dev, st, out = _run(tmp_path, "dev", {"WASTE_METAL_MOE": "1", "WASTE_CACHE_MB": "8",
                                          "WARP_CUDA_DEVICE_MIN_KB": "0"})
    assert "backend CUDA sm_100a" in out, out
    assert st is not None and st["mvq_device"] > 0 and st["vq3r_jobs"] > 0, st
    _logitcmp(dev, cpu)
