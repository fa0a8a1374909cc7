"""Build libheatkv.so in-tree with nvcc for sm_100a.

``python -m heatkv_b200.build`` compiles every ``csrc/*.cu`` and ``csrc/*.cpp`` (host code) (whole-program device code: kernels
receive the device status word's address as a parameter, and ``setmaxnreg`` register splits are
only honoured without relocatable device code) and links ``heatkv_b200/libheatkv.so``. Objects go to
``heatkv_b200/_build/``; a file is recompiled only when it or a header changed. The build needs no
GPU: nvcc cross-compiles for ``-gencode arch=compute_100a,code=sm_100a``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libheatkv.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
              "--expt-relaxed-constexpr", "-I", os.path.join(REPO, "include"), "-I", CSRC]


def nvcc() -> str:
    path = shutil.which("nvcc")
    if path is None:
        cand = "/usr/local/cuda/bin/nvcc"
        if os.path.exists(cand):
            return cand
        raise RuntimeError("nvcc not found; libheatkv.so cannot be built")
    return path


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(REPO, "include", "*.h"))


def _stale(obj: str, src: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src] + _headers())


def _compile(src: str, obj: str, verbose: bool, extra) -> None:
    cmd = [nvcc()] + ARCH + NVCC_FLAGS + list(extra) + ["-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{res.stdout}{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    objs = [os.path.join(BUILD, os.path.splitext(os.path.basename(s))[0] + ".o") for s in srcs]
    todo = [(s, o) for s, o in zip(srcs, objs) if force or _stale(o, s)]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as ex:
            list(ex.map(lambda so: _compile(so[0], so[1], verbose, extra), todo))
    if todo or force or not os.path.exists(LIB) or \
            any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc()] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-cudart", "static",
                                 "-o", tmp] + objs
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link of libheatkv.so failed:\n{res.stdout}{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    args = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if args.ptxas_info else []
    print(build(force=args.force or args.ptxas_info, verbose=args.verbose or args.ptxas_info,
                extra=extra))


if __name__ == "__main__":
    main(sys.argv[1:])
