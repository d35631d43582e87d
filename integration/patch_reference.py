"""Compiles the reference's own decode loops against the B200 sampler.

Copies main.cu and python/bindings.cu from a reference tree into
integration/_build/ (never into the repository), makes the one edit a
maintainer would make -- the sampler include becomes qs_sampler_compat.h --
and compiles each with nvcc for sm_100a (-c: the model, tokenizer and
pybind11 parts come from the reference tree as they are).  Success shows
that the loops that call build_sampler / sample / reset_sampler_history /
free_sampler and write the Sampler fields (main.cu:136-139, 296-303;
python/bindings.cu:91-100, 170, 193, 202, 213-238) build unchanged on the
C ABI.

    python integration/patch_reference.py <reference tree>
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
OUT = os.path.join(HERE, "_build")

EDITS = {
    "main.cu": ('#include "sampler.h"', '#include "qs_sampler_compat.h"'),
    "bindings.cu": ('#include "../sampler.h"', '#include "qs_sampler_compat.h"'),
}


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def patch(ref: str) -> dict:
    os.makedirs(OUT, exist_ok=True)
    srcs = {"main.cu": os.path.join(ref, "main.cu"),
            "bindings.cu": os.path.join(ref, "python", "bindings.cu")}
    out = {}
    for name, src in srcs.items():
        text = open(src).read()
        old, new = EDITS[name]
        if text.count(old) != 1:
            raise RuntimeError(f"{name}: expected one '{old}'")
        dst = os.path.join(OUT, "patched_" + name)
        with open(dst, "w") as f:
            f.write(text.replace(old, new))
        out[name] = dst
    return out


def compile_all(ref: str) -> dict:
    files = patch(ref)
    base = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-c",
            "-I", HERE, "-I", os.path.join(ROOT, "include"), "-I", ref]
    results = {}
    for name, path in files.items():
        cmd = list(base)
        if name == "bindings.cu":
            import sysconfig

            import pybind11
            cmd += ["-I", os.path.join(ref, "python"), "-I", pybind11.get_include(),
                    "-I", sysconfig.get_paths()["include"], "-Xcompiler", "-fPIC"]
        cmd += [path, "-o", path[:-3] + ".o"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        results[name] = (r.returncode, r.stderr[-4000:])
    return results


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    res = compile_all(sys.argv[1])
    for name, (rc, err) in res.items():
        print(name, "ok" if rc == 0 else f"failed:\n{err}")
    sys.exit(0 if all(rc == 0 for rc, _ in res.values()) else 1)
