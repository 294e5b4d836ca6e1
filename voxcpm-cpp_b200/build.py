#!/usr/bin/env python3
"""Builds libvcpm_b200.so (the C-ABI hot-path library) for sm_100a, in-tree.

Every csrc/*.cu compiles to an object under _build/ (in parallel), then one
shared library is linked next to this file.  Flags: sm_100a only, -O3,
-lineinfo, and -ffp-contract=off for host code so the host-built tables
(rotary cos/sin, time sinusoids) round exactly as written.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libvcpm_b200.so")
ROOT = os.path.dirname(HERE)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
HOST_CXX = shutil.which("g++", path="/usr/bin") or "g++"


def nvcc() -> str:
    for p in (os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"), shutil.which("nvcc")):
        if p and os.path.exists(p):
            return p
    raise RuntimeError("nvcc not found")


def flags(verbose_ptxas: bool = False) -> list[str]:
    f = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-ccbin", HOST_CXX,
                "-Xcompiler", "-fPIC,-ffp-contract=off,-O2", "-I", os.path.join(ROOT, "include")]
    if verbose_ptxas:
        f += ["-Xptxas", "-v"]
    return f


def _compile(src: str, verbose: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    deps = [src] + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith(".cuh")]
    deps.append(os.path.join(ROOT, "include", "vcpm_b200.h"))
    if os.path.exists(obj) and all(os.path.getmtime(obj) >= os.path.getmtime(d) for d in deps) and not verbose:
        return obj, ""
    cmd = [nvcc()] + flags(verbose) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(verbose: bool = False, jobs: int = 8) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), srcs))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            sys.stderr.write(log)
    if not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-ccbin", HOST_CXX, "-o", LIB] + objs + ["-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    build_host()
    return LIB


HOST_SRC = os.path.join(HERE, "host", "vcpm_gen_run.c")
HOST_BIN = os.path.join(HERE, "host", "vcpm_gen_run")


def build_host() -> str:
    """The C11 host driver (host/vcpm_gen_run.c): compiled as plain C with
    warnings as errors against include/vcpm_b200.h alone and linked to the
    library above (rpath: the library's directory)."""
    hdr = os.path.join(ROOT, "include", "vcpm_b200.h")
    if os.path.exists(HOST_BIN) and all(os.path.getmtime(HOST_BIN) >= os.path.getmtime(d)
                                        for d in (HOST_SRC, hdr, LIB)):
        return HOST_BIN
    cc = shutil.which("gcc", path="/usr/bin") or "gcc"
    cmd = [cc, "-std=c11", "-O2", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", os.path.join(ROOT, "include"),
           HOST_SRC, "-o", HOST_BIN, "-L", HERE, "-lvcpm_b200", "-Wl,-rpath," + HERE, "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"host driver build failed:\n{r.stdout}\n{r.stderr}")
    return HOST_BIN


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
