"""Builds librace_b200.so in-tree with nvcc for sm_100a.

    python -m race_attention_b200.build      (or __graft_entry__.build())

The three translation units compile in parallel; the result lands next to
this file so it travels with the source tree.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "librace_b200.so")
SOURCES = ["race_capi.cu", "race_f32_d32.cu", "race_f32_d64.cu", "race_bf16_d32.cu",
           "race_bf16_d64.cu", "race_probs.cu", "race_comm.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    hdr = os.path.join(ROOT, "include", "race_b200.h")
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [hdr, os.path.abspath(__file__)]
    return any(os.path.getmtime(p) > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return OUT
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    cc = nvcc()

    def compile_one(src):
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        cmd = [cc, *ARCH, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr}")
        if verbose and r.stderr:
            print(r.stderr, file=sys.stderr)
        return obj

    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if not f.endswith(".cu")]
    hdrs.append(os.path.join(ROOT, "include", "race_b200.h"))
    newest_hdr = max(os.path.getmtime(h) for h in hdrs)

    def fresh(src):
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        return (not force and os.path.exists(obj) and
                os.path.getmtime(obj) > max(newest_hdr, os.path.getmtime(os.path.join(CSRC, src))))

    todo = [s for s in SOURCES if not fresh(s)]
    with cf.ThreadPoolExecutor(max(1, len(todo))) as ex:
        list(ex.map(compile_one, todo))
    objs = [os.path.join(objdir, s.replace(".cu", ".o")) for s in SOURCES]
    tmp = OUT + ".tmp"
    cmd = [cc, *ARCH, "-shared", "-o", tmp, *objs, "-ldl"]   # cudart linked statically
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
