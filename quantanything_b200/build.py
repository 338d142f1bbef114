"""Builds the CUDA kernel library ``quantanything_b200/lib/libqa_kernels.so``.

Every ``csrc/*.cu`` is compiled for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``) and linked with the static CUDA runtime,
so the shared object carries no dependency on the CUDA runtime bundled
with PyTorch and loads in any process of this image.  The driver's
tensor-map encoder is resolved at run time (``cudaGetDriverEntryPoint``),
so the library also loads on machines without a GPU driver (calls then
fail with a recorded error).

Usage: ``python -m quantanything_b200.build [--force] [--jobs N]``
"""

import argparse
import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "lib" / "_obj"
LIB = PKG / "lib" / "libqa_kernels.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", f"-I{INCLUDE}"]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found")
    return path


def _host_compiler():
    # The image's $CXX wrapper lacks some runtime specs; nvcc gets the system
    # g++ explicitly.
    return ["-ccbin", "/usr/bin/g++"] if Path("/usr/bin/g++").exists() else []


def _stale(obj, src, deps):
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(d.stat().st_mtime > t for d in deps)


def build(force=False, jobs=None, verbose=False):
    """Compiles the sources that changed and links the library; returns its path."""
    BUILD.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    todo = []
    objs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, src, headers):
            todo.append((src, obj))

    def compile_one(item):
        src, obj = item
        cmd = [nvcc(), *_host_compiler(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{proc.stderr}")
        if verbose:
            print("compiled", src.name)

    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as pool:
        list(pool.map(compile_one, todo))
    if todo or force or not LIB.exists():
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *_host_compiler(), *ARCH, "-shared", "-cudart", "static",
               *map(str, objs), "-o", str(tmp)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose=True))


if __name__ == "__main__":
    main()
