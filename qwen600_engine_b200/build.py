"""Builds the sampler's CUDA library in-tree for sm_100a.

Produces qwen600_engine_b200/libqwen600_sampler.so from csrc/*.cu with nvcc
(no GPU needed: nvcc cross-compiles).  --fmad=false keeps every fp32
multiply and add separately rounded, as the reference host sampler computes
them; -lineinfo keeps profiler source correlation.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libqwen600_sampler.so")
SOURCES = ["qs_row.cu", "qs_row_wide.cu", "qs_ties.cu", "qs_sort.cu", "qs_api.cu", "qs_static.cu", "qs_lmhead.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "--fmad=false", "-std=c++17", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "-I", os.path.join(ROOT, "include"), "-I", CSRC,
         "-I", OUT_DIR]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def exp_table(verbose: bool = False) -> str:
    """Generates _build/qs_exp_table.inc: the inputs where the host libm's
    expf (what the reference sampler calls) rounds differently from
    qs_exp_rn.  Takes about a minute; redone only when its sources change."""
    os.makedirs(OUT_DIR, exist_ok=True)
    inc = os.path.join(OUT_DIR, "qs_exp_table.inc")
    gen_src = os.path.join(CSRC, "qs_exp_table.c")
    deps = [gen_src, os.path.join(CSRC, "qs_exp.h")]
    if not _stale(inc, deps):
        return inc
    exe = os.path.join(OUT_DIR, "qs_exp_table")
    cc = shutil.which("gcc") or "cc"
    flags = ["-O2", "-ffp-contract=off"]
    try:
        if " fma " in open("/proc/cpuinfo").read():
            flags.append("-mfma")  # hardware fma: same IEEE result, faster scan
    except OSError:
        pass
    r = subprocess.run([cc] + flags + ["-I", CSRC, "-o", exe, gen_src, "-lm"],
                       capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compiling qs_exp_table.c failed:\n{r.stderr}")
    tmp = inc + ".tmp"
    r = subprocess.run([exe, tmp], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"qs_exp_table failed:\n{r.stderr}")
    os.replace(tmp, inc)
    if verbose:
        print(r.stdout.strip())
    return inc


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    table = exp_table(verbose)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(table)
    headers.append(os.path.join(ROOT, "include", "qwen600_sampler.h"))
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OUT_DIR, src.replace(".cu", ".o"))
        objs.append(o)
        if force or ptxas_info or _stale(o, [s, __file__] + headers):
            cmd = [nvcc()] + ARCH + FLAGS + ["-c", s, "-o", o]
            if ptxas_info:
                cmd += ["-Xptxas", "-v"]
            if verbose:
                print(" ".join(cmd))
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
            if ptxas_info or verbose:
                sys.stderr.write(r.stderr)
    if force or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    build_integration(verbose, force)
    return LIB


INTEG = os.path.join(ROOT, "integration")
DEMO_LIB = os.path.join(INTEG, "libqs_decode_demo.so")


def build_integration(verbose: bool = False, force: bool = False) -> str:
    """integration/libqs_decode_demo.so: a decode loop written against the
    reference sampler's interface (integration/qs_sampler_compat.h), linked to
    the sampler library."""
    src = os.path.join(INTEG, "decode_demo.cu")
    deps = [src, os.path.join(INTEG, "qs_sampler_compat.h"), os.path.join(ROOT, "include", "qwen600_sampler.h"),
            LIB, __file__]
    if not force and not _stale(DEMO_LIB, deps):
        return DEMO_LIB
    cmd = [nvcc()] + ARCH + ["-O2", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
                             "-Xcompiler", "-fvisibility=hidden", "-I", os.path.join(ROOT, "include"), "-I", INTEG,
                             src, "-o", DEMO_LIB, "-L", HERE, "-lqwen600_sampler",
                             "-Xlinker", "-rpath,$ORIGIN/../qwen600_engine_b200"]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"building the decode demo failed:\n{r.stderr}")
    return DEMO_LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_info="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
