"""Builds libzealot_attn.so in-tree with nvcc for sm_100a.

    python zealot_b200/build.py            # incremental
    python zealot_b200/build.py --force    # rebuild everything

(run as a file, not with -m: importing the package loads the library, which
does not exist yet on a fresh checkout)

Every .cu / .cc file under zealot_b200/csrc is compiled with
-gencode arch=compute_100a,code=sm_100a and linked into
zealot_b200/libzealot_attn.so (static CUDA runtime, no libcuda link: the
driver entry points are resolved at run time, so the library also loads on a
machine without a GPU driver).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libzealot_attn.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
          "-ccbin", "/usr/bin/g++", f"-I{INCLUDE}", "-I/usr/include"]


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cc")))


def _headers_mtime() -> float:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(INCLUDE, "zealot_attn.h"))
    return max(os.path.getmtime(h) for h in hs)


def _compile(src: str, force: bool, verbose_ptxas: bool) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if (not force and os.path.exists(obj) and os.path.getmtime(obj) >= os.path.getmtime(src)
            and os.path.getmtime(obj) >= _headers_mtime()):
        return obj
    cmd = [NVCC, *ARCH, *COMMON, "-c", src, "-o", obj]
    if src.endswith(".cc"):
        cmd[1:1] = ["-x", "cu"]
    if verbose_ptxas and src.endswith(".cu"):
        cmd.append("-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose_ptxas:
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose_ptxas), srcs))
    if (force or not os.path.exists(LIB)
            or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs)):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-ccbin", "/usr/bin/g++", "-o", LIB,
               *objs, "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v resource usage")
    a = ap.parse_args()
    print(build(force=a.force, verbose_ptxas=a.ptxas))
