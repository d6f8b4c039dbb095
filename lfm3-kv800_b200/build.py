"""Build the CUDA library of the 800h hot path for B200 (sm_100a):

    python lfm3-kv800_b200/build.py            # -> lfm3-kv800_b200/lfm3_kv800/_lib/libkv800_b200.so

nvcc cross-compiles without a GPU.  Every csrc/*.cu file is compiled to an object (in parallel) and linked into one
shared library with a plain C ABI (include/kv800_b200.h); the CUDA runtime is linked statically, so the library only
needs the driver.  The library is rebuilt when a source or header is newer than it."""
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "lfm3_kv800", "_lib")
LIB = os.path.join(OUT_DIR, "libkv800_b200.so")
BUILD = os.path.join(HERE, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden", "-Xptxas", "-v",
                  "-I" + os.path.join(ROOT, "include")]


def nvcc():
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found (CUDA 12.9 toolkit expected)")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return _sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h")) + [
        os.path.abspath(__file__)]


def up_to_date():
    return os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(p) for p in _deps())


def _compile(src):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    r = subprocess.run([nvcc()] + NVFLAGS + ["-c", src, "-o", obj], capture_output=True, text=True)
    return src, obj, r.returncode, r.stdout + r.stderr


def build(force=False, verbose=False):
    if not force and up_to_date():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(OUT_DIR, exist_ok=True)
    objs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for src, obj, rc, log in ex.map(_compile, _sources()):
            if rc:
                raise RuntimeError(f"nvcc failed on {src}:\n{log}")
            if verbose:
                print(log, end="")
            objs.append(obj)
    tmp = LIB + ".tmp"
    r = subprocess.run([nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs,
                       capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"link failed:\n{r.stdout}{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
