"""Build libkvr_b200.so (the C-ABI engine library) in-tree for sm_100a.

    python -m budgeted_kv_cache_repair_b200.build [--jobs N] [--force]

Each ``csrc/*.cu`` compiles to an object with
``-gencode arch=compute_100a,code=sm_100a``; the objects link into
``lib/libkvr_b200.so`` next to this file. Rebuilds only when a source or header
is newer than the library. nvcc cross-compiles, so this runs without a GPU.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import glob
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
LIBRARY = os.path.join(LIBDIR, "libkvr_b200.so")
INCLUDE = os.path.join(ROOT, "include")
CUDA_LIB = "/usr/local/cuda/lib64"  # fallback search path for libcublas when torch has not loaded it

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "-I", INCLUDE]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(found):
        raise RuntimeError("nvcc not found; the B200 engine needs the CUDA toolkit to build")
    return found


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return (_sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(INCLUDE, "*.h")) + [__file__])


def up_to_date() -> bool:
    if not os.path.exists(LIBRARY):
        return False
    built = os.path.getmtime(LIBRARY)
    return all(os.path.getmtime(p) <= built for p in _deps())


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIBRARY
    os.makedirs(LIBDIR, exist_ok=True)
    objdir = os.path.join(LIBDIR, "obj")
    os.makedirs(objdir, exist_ok=True)
    compiler = nvcc()

    def compile_one(src):
        obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
        cmd = [compiler, *ARCH, *FLAGS, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode:
            raise RuntimeError(f"nvcc failed for {src}:\n{proc.stdout}\n{proc.stderr}")
        return obj, proc.stderr

    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as pool:
        results = list(pool.map(compile_one, _sources()))
    if verbose:
        for _, log in results:
            print(log)
    tmp = LIBRARY + ".tmp"
    cmd = [compiler, *ARCH, "-shared", "-o", tmp, *[o for o, _ in results], "-lcudart", "-lcublas", "-lnccl",
           "-Xlinker", "-rpath=" + CUDA_LIB]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode:
        raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, LIBRARY)
    return LIBRARY


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int, default=None)
    parser.add_argument("--verbose", action="store_true", help="print ptxas register/spill reports")
    args = parser.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose=args.verbose))


if __name__ == "__main__":
    main()
