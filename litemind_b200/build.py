"""Builds liblitemind_b200.so in-tree with nvcc for sm_100a.

    python -m litemind_b200.build            # incremental
    python -m litemind_b200.build --force    # rebuild everything

Objects go to litemind_b200/_build/; the shared library to
litemind_b200/liblitemind_b200.so, next to the Python loader that opens it.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "liblitemind_b200.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
              "-Xptxas", "-v", f"-I{INCLUDE}", f"-I{CSRC}"]
CXX_FLAGS = ["-O3", "-std=c++20", "-fPIC", "-Wall", "-Wextra", f"-I{INCLUDE}", f"-I{CSRC}"]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _cuda_home() -> str:
    return os.path.dirname(os.path.dirname(os.path.realpath(_nvcc())))


def sources() -> list[str]:
    out = []
    for sub in ("", "host"):
        d = os.path.join(CSRC, sub)
        if not os.path.isdir(d):
            continue
        for name in sorted(os.listdir(d)):
            if name.endswith((".cu", ".cpp")):
                out.append(os.path.join(d, name))
    return out


def _headers() -> list[str]:
    hs = []
    for d in (CSRC, os.path.join(CSRC, "host"), INCLUDE, os.path.join(INCLUDE, "litemind_b200")):
        if os.path.isdir(d):
            hs += [os.path.join(d, n) for n in os.listdir(d) if n.endswith((".h", ".hpp", ".cuh"))]
    return hs


def _compile(src: str, force: bool, verbose: bool) -> str:
    rel = os.path.relpath(src, CSRC).replace(os.sep, "_")
    obj = os.path.join(BUILD, rel + ".o")
    newest_header = max((os.path.getmtime(h) for h in _headers()), default=0)
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), newest_header):
        return obj
    cuda_inc = os.path.join(_cuda_home(), "include")
    if src.endswith(".cu"):
        cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    else:
        cmd = ["g++", *CXX_FLAGS, f"-I{cuda_inc}", "-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stderr or res.stdout):
        log = os.path.join(BUILD, rel + ".log")
        with open(log, "w") as f:
            f.write(res.stdout + res.stderr)
    return obj


def build(force: bool = False, verbose: bool = True) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objs = list(pool.map(lambda s: _compile(s, force, verbose), srcs))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [_nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-cudart", "static", "-lpthread", "-ldl"]  # NCCL: dlopen
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
