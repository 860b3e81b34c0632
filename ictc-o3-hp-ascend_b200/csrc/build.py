"""Build libictc_cuda.so for sm_100a from the CUDA sources in this folder.

Each .cu file is compiled to an object in parallel, then linked into
``ictc_o3/backends/cuda/libictc_cuda.so`` beside the Python package that
loads it.  The CUDA runtime is linked statically, so the library carries no
dependency on a particular libcudart soname.

    python build.py [--force] [--verbose]
"""
import argparse
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
INCLUDE = os.path.join(REPO, "include")
OBJDIR = os.path.join(PKG, "_build")
OUTPUT = os.path.join(PKG, "ictc_o3", "backends", "cuda", "libictc_cuda.so")
NVCC = os.environ.get("NVCC", "nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
         "-Xcompiler", "-fPIC", "-I" + INCLUDE, "-I" + HERE]


def sources():
    return sorted(f for f in os.listdir(HERE) if f.endswith(".cu"))


def _deps_mtime():
    stamps = [os.path.getmtime(os.path.join(HERE, f)) for f in os.listdir(HERE)
              if f.endswith((".cuh", ".h"))]
    stamps += [os.path.getmtime(os.path.join(INCLUDE, f)) for f in os.listdir(INCLUDE)]
    return max(stamps) if stamps else 0.0


def _compile(src, force, verbose):
    obj = os.path.join(OBJDIR, src[:-3] + ".o")
    path = os.path.join(HERE, src)
    if (not force and os.path.exists(obj)
            and os.path.getmtime(obj) >= max(os.path.getmtime(path), _deps_mtime())):
        return obj
    cmd = [NVCC, *FLAGS, "-c", path, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{proc.stderr}")
    if verbose:
        sys.stderr.write(proc.stderr)
    return obj


def build(force=False, verbose=False):
    os.makedirs(OBJDIR, exist_ok=True)
    srcs = sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 1))) as pool:
        objs = list(pool.map(lambda s: _compile(s, force, verbose), srcs))
    if (not force and os.path.exists(OUTPUT)
            and os.path.getmtime(OUTPUT) >= max(os.path.getmtime(o) for o in objs)):
        return OUTPUT
    tmp = OUTPUT + ".tmp"
    cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static",
           *objs, "-o", tmp]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link failed:\n{proc.stderr}")
    os.replace(tmp, OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(args.force, args.verbose))
