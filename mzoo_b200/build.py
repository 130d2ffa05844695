"""Build ``libmzb200.so`` in-tree with nvcc for sm_100a.

``python -m mzoo_b200.build`` (or ``build()``) compiles every ``csrc/*.cu`` to an object
under ``_build/`` in parallel and links them into ``mzoo_b200/libmzb200.so``.  The CUDA
runtime is linked statically and the driver is reached only through the runtime, so the
library loads (and its symbols can be listed) on a host without a GPU.
"""

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT = os.path.join(PKG, "libmzb200.so")
BUILD = os.path.join(ROOT, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                     "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources() -> list:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps() -> list:
    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hdrs + [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(p) <= t for p in _sources() + _deps() + [__file__])


def _compile(src: str, extra: list) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc()] + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip() and os.environ.get("MZB_BUILD_VERBOSE"):
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose: bool = False, extra: list | None = None) -> str:
    """Compile and link; returns the path of the shared library."""
    if not force and up_to_date():
        return OUT
    os.makedirs(BUILD, exist_ok=True)
    extra = list(extra or [])
    if verbose:
        extra += ["-Xptxas", "-v"]
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), srcs))
    tmp = OUT + ".tmp"
    cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
