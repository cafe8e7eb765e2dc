"""Builds the sm_100a kernel library in-tree: llama2_b200/libllama2_b200.so.

    python -m llama2_b200.build [-v] [--force]

Every .cu file in csrc/ is compiled by nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a), the host-only .cpp files by the
host compiler with -ffp-contract=off, and everything is linked into one
shared library with the CUDA runtime linked statically (so the library does
not depend on which libcudart the calling process has loaded). Objects are
rebuilt only when a source or header is newer.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libllama2_b200.so")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xcompiler", "-ffp-contract=off", f"-I{INCLUDE}", f"-I{CSRC}"] + ARCH
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-ffp-contract=off", "-fno-fast-math", f"-I{INCLUDE}",
             f"-I{CUDA_HOME}/include"]


def _sources():
    out = []
    for name in sorted(os.listdir(CSRC)):
        if name.endswith((".cu", ".cpp")):
            out.append(os.path.join(CSRC, name))
    return out


def _headers():
    hs = [os.path.join(INCLUDE, h) for h in os.listdir(INCLUDE) if h.endswith(".h")]
    hs += [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h"))]
    return hs


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, verbose):
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if src.endswith(".cu"):
        cmd = [NVCC, *NVCC_FLAGS, "-c", src, "-o", obj]
        if verbose:
            cmd += ["-Xptxas", "-v"]
    else:
        cmd = [os.environ.get("CXX", "g++"), *CXX_FLAGS, "-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return obj, (res.stdout + res.stderr) if verbose else ""


def build(verbose: bool = False, force: bool = False) -> str:
    if not os.path.exists(NVCC):
        raise RuntimeError(f"nvcc not found at {NVCC}")
    os.makedirs(OBJ, exist_ok=True)
    srcs = _sources()
    headers = _headers()
    todo = [s for s in srcs if force or _stale(os.path.join(OBJ, os.path.basename(s) + ".o"), [s, *headers])]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
            for obj, log in ex.map(lambda s: _compile(s, verbose), todo):
                if log:
                    print(f"== {os.path.basename(obj)}\n{log}", file=sys.stderr)
    objs = [os.path.join(OBJ, os.path.basename(s) + ".o") for s in srcs]
    if force or todo or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [NVCC, "-shared", *ARCH, "-o", tmp, *objs, "-cudart", "static"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        shutil.move(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas resource usage")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(verbose=args.verbose, force=args.force))


if __name__ == "__main__":
    main()
