"""Build the sm_100a backend library in-tree: odiengine_b200/libodi_cuda.so.

    python -m odiengine_b200.build          # or odiengine_b200.build.build()

Each .cu file under csrc/ is compiled with
``nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` and linked
into one shared library with the static CUDA runtime, so the .so has no
dependency beyond the driver.  Objects go to odiengine_b200/_build/.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libodi_cuda.so")
BUILD = os.path.join(HERE, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
           "--expt-relaxed-constexpr", "-Xptxas", "-v,-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise FileNotFoundError("nvcc not found")


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _compile(src: str) -> tuple[str, str]:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc(), *ARCH, *NVFLAGS, "-I", os.path.join(HERE, "..", "include"), "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(verbose: bool = False) -> str:
    """Compile every .cu file and link libodi_cuda.so.  Returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(_compile, srcs))
    if verbose:
        for _, log in results:
            sys.stderr.write(log)
    objs = [o for o, _ in results]
    tmp = OUT + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
