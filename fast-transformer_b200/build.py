"""Build libfastb200.so in-tree for sm_100a (B200).

    python fast-transformer_b200/build.py [--force] [--jobs N]

Every csrc/*.cu is compiled with nvcc (-gencode arch=compute_100a,code=sm_100a -lineinfo)
into _build/, then linked into fast-transformer_b200/libfastb200.so with a static CUDA
runtime, so the library depends only on the driver. Objects are rebuilt when their source,
a header, or this script changes.
"""

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBRARY = os.path.join(HERE, "libfastb200.so")
HEADERS = [os.path.join(ROOT, "include", "fastb200.h")]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include")]


def nvcc():
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(found):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libfastb200.so")
    return found


def sources():
    return sorted(os.path.join(CSRC, name) for name in os.listdir(CSRC) if name.endswith(".cu"))


def _stamp(paths):
    return max(os.path.getmtime(p) for p in paths)


def _compile(src, verbose):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    deps = [src, __file__] + HEADERS + [
        os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h"))
    ]
    if os.path.exists(obj) and os.path.getmtime(obj) >= _stamp(deps):
        return obj, ""
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{proc.stderr}")
    return obj, proc.stderr


def build(force=False, jobs=None, verbose=False):
    """Compile and link; returns the library path."""
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    if force:
        for name in os.listdir(BUILD):
            os.remove(os.path.join(BUILD, name))
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with concurrent.futures.ThreadPoolExecutor(jobs) as pool:
        results = list(pool.map(lambda s: _compile(s, verbose), srcs))
    objs = [obj for obj, _ in results]
    if verbose:
        for _, log in results:
            if log:
                sys.stderr.write(log)
    if force or not os.path.exists(LIBRARY) or os.path.getmtime(LIBRARY) < _stamp(objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", LIBRARY, *objs]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stderr}")
    return LIBRARY


if __name__ == "__main__":
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int)
    parser.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    args = parser.parse_args()
    print(build(args.force, args.jobs, args.verbose))
