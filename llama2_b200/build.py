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
CPP = os.path.join(PKG, "cpp")
INCLUDE = os.path.join(ROOT, "include")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libllama2_b200.so")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xcompiler", "-ffp-contract=off", f"-I{INCLUDE}", f"-I{CSRC}"] + ARCH
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-ffp-contract=off", "-fno-fast-math", f"-I{INCLUDE}",
             f"-I{CUDA_HOME}/include", f"-I{os.path.join(CPP, 'include')}"]
DROPIN_TEST = os.path.join(CPP, "tests", "test_dropin")


def _sources():
    out = []
    for name in sorted(os.listdir(CSRC)):
        if name.endswith((".cu", ".cpp")):
            out.append(os.path.join(CSRC, name))
    out.append(os.path.join(CPP, "src", "dropin.cpp"))  # C++ operator API over the C ABI
    return out


def _headers():
    hs = [os.path.join(INCLUDE, h) for h in os.listdir(INCLUDE) if h.endswith(".h")]
    hs += [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h"))]
    for sub in ("common", "core", "kernel"):
        d = os.path.join(CPP, "include", sub)
        hs += [os.path.join(d, h) for h in os.listdir(d)]
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
        # CUDA runtime linked statically and its symbols kept private, so a
        # caller's own libcudart can neither interpose on nor clash with it.
        cmd = [NVCC, "-shared", *ARCH, "-o", tmp, *objs, "-cudart", "static", "-Xlinker", "--exclude-libs,ALL"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        shutil.move(tmp, LIB)
    return LIB


def build_dropin_test() -> str:
    """The C++ test program of the drop-in API (test infrastructure): links the
    library, the C oracle (expectations) and the CUDA runtime."""
    lib = LIB
    if not os.path.exists(lib):
        lib = build()
    oracle_dir = os.path.join(ROOT, "oracle")
    subprocess.run(["make", "-s", "-C", oracle_dir, "liboracle.so"], check=True)
    src = os.path.join(CPP, "tests", "test_dropin.cpp")
    if not _stale(DROPIN_TEST, [src, lib, *_headers()]):
        return DROPIN_TEST
    cmd = [os.environ.get("CXX", "g++"), "-std=c++17", "-O2", f"-I{INCLUDE}", f"-I{os.path.join(CPP, 'include')}",
           f"-I{CUDA_HOME}/include", src, "-o", DROPIN_TEST, f"-L{PKG}", "-lllama2_b200", f"-L{oracle_dir}",
           "-loracle", f"-L{CUDA_HOME}/lib64", "-lcudart", "-Wl,-rpath,$ORIGIN/../..",
           "-Wl,-rpath,$ORIGIN/../../../oracle", f"-Wl,-rpath,{CUDA_HOME}/lib64"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"drop-in test build failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return DROPIN_TEST


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas resource usage")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(verbose=args.verbose, force=args.force))


if __name__ == "__main__":
    main()
