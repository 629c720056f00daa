"""Builds libhypno_cuda.so in-tree for sm_100a with nvcc.

Usage: python -m hypno_b200.build   (or hypno_b200.build.build())
Each .cu under csrc/ is compiled with
  -gencode arch=compute_100a,code=sm_100a -lineinfo -O3
and linked into hypno_b200/libhypno_cuda.so (static cudart, hidden symbols
except the extern "C" entry points declared in include/hypno_cuda.h).
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libhypno_cuda.so")
BUILD = os.path.join(HERE, "_build")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden,-fopenmp",
         "-Xptxas", "-warn-spills", "--expt-relaxed-constexpr", "-ccbin", "g++"]


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _newest_input():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    files.append(os.path.join(HERE, "..", "include", "hypno_cuda.h"))
    files.append(os.path.abspath(__file__))
    return max(os.path.getmtime(f) for f in files)


def build(force=False, verbose=False):
    """Compiles every CUDA source and links the shared library; skips the work
    when the library is newer than every input."""
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= _newest_input():
        return OUT
    os.makedirs(BUILD, exist_ok=True)
    env = dict(os.environ)
    env.pop("CC", None)
    env.pop("CXX", None)

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True, env=env)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, file=sys.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = OUT + ".tmp"
    cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-Xcompiler", "-fopenmp", "-ccbin", "g++", "-lgomp"]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
