"""Build libwarp_cuda.so in-tree with nvcc for sm_100a.

    python -m warp_b200.build            # build if any source is newer
    python -m warp_b200.build --force    # rebuild everything

Objects go to warp_b200/_build/, the library to warp_b200/lib/.  The build is
plain nvcc (no torch extension machinery): the library's ABI is C, declared in
include/warp_cuda.h, and it links only against the CUDA runtime.
"""
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libwarp_cuda.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
    "-DWARP_BUILD",
]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _newest_header():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(ROOT, "include", "warp_cuda.h"))
    return max(os.path.getmtime(h) for h in hs if os.path.exists(h))


def build(force=False, verbose=False, ptxas_v=False):
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    nv = nvcc()
    hdr = _newest_header()
    jobs = []
    objs = []
    for f in sources():
        src = os.path.join(CSRC, f)
        obj = os.path.join(OBJ, f[:-3] + ".o")
        objs.append(obj)
        stale = force or not os.path.exists(obj) or \
            os.path.getmtime(obj) < max(os.path.getmtime(src), hdr)
        if stale:
            cmd = [nv] + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_v else []) + \
                ["-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
            jobs.append((f, cmd))

    def run(job):
        f, cmd = job
        r = subprocess.run(cmd, capture_output=True, text=True)
        return f, r

    failed = []
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for f, r in ex.map(run, jobs):
            out = (r.stdout + r.stderr).strip()
            if r.returncode != 0:
                failed.append(f)
                sys.stderr.write(f"[warp_b200] nvcc failed on {f}:\n{out}\n")
            elif out and (verbose or ptxas_v):
                sys.stderr.write(f"[warp_b200] {f}:\n{out}\n")
    if failed:
        raise RuntimeError("nvcc failed: " + ", ".join(failed))
    lib_stale = force or jobs or not os.path.exists(LIB) or \
        os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs)
    if lib_stale:
        cmd = [nv] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv,
          ptxas_v="--ptxas" in sys.argv)
    print(LIB)
