"""Build ``liblb_b200.so`` (the C-ABI CUDA library) in-tree with nvcc for sm_100a.

``python -m layerbatch_b200.build`` compiles every ``csrc/*.cu`` to an object in parallel
and links them into ``layerbatch_b200/liblb_b200.so`` with the CUDA runtime linked
statically (the library needs no libcudart/libcuda at link time; the driver's tensor-map
encoder is resolved at run time).  Cross-compiles without a GPU.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD_DIR = os.path.join(HERE, "_build")
LIB_PATH = os.path.join(HERE, "liblb_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-v"]


def nvcc_path() -> str:
    cand = [os.environ.get("NVCC", ""), shutil.which("nvcc") or "", "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found (set NVCC or add /usr/local/cuda/bin to PATH)")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _needs_rebuild(obj, src):
    if not os.path.exists(obj):
        return True
    deps = [src] + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
    deps += glob.glob(os.path.join(os.path.dirname(HERE), "include", "*.h"))
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, obj, log):
    cmd = [nvcc_path(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    with open(log, "w") as f:
        f.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stderr[-6000:]}")
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD_DIR, exist_ok=True)
    srcs = sources()
    objs = [os.path.join(BUILD_DIR, os.path.basename(s)[:-3] + ".o") for s in srcs]
    todo = [(s, o) for s, o in zip(srcs, objs) if force or _needs_rebuild(o, s)]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            futs = [ex.submit(_compile, s, o, o + ".log") for s, o in todo]
            for f in futs:
                f.result()
    if force or todo or not os.path.exists(LIB_PATH):
        tmp = LIB_PATH + ".tmp"
        cmd = [nvcc_path(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stderr[-4000:])
        os.replace(tmp, LIB_PATH)
    if verbose:
        for o in objs:
            with open(o + ".log") as f:
                print(f.read())
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
