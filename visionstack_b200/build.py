"""Build the sm_100a shared library ``libgdn_b200.so`` in-tree with nvcc.

    python -m visionstack_b200.build [--force]

Cross-compiles without a GPU.  The library is written next to this file so it
travels with the source tree.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
REPO = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libgdn_b200.so")
SOURCES = ["gdn_capi.cu", "gdn_decode.cu", "gdn_decode_tma.cu", "gdn_prefill.cu", "gdn_conv.cu",
           "gdn_umma_selftest.cu", "gdn_prefill_tc.cu", "gdn_tmap.cu", "gdn_slots.cu",
           "gdn_prefill_prep.cu", "gdn_prefill_seq.cu", "gdn_prefill_static.cu", "stack_attn_decode.cu",
           "gdn_functional.cu", "gdn_prefill_fused.cu", "gdn_peer_allreduce.cu",
           "stack_ops.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _inputs():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".h"))]
    files.append(os.path.join(REPO, "include", "gdn_b200.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    common = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", os.path.join(REPO, "include"),
                     "--expt-relaxed-constexpr"]
    if verbose:
        common += ["-Xptxas", "-v"]
    procs = []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        cmd = [nvcc()] + common + ["-c", os.path.join(CSRC, src), "-o", obj]
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    for cmd, pr in procs:
        out, _ = pr.communicate()
        if verbose or pr.returncode != 0:
            sys.stderr.write(out.decode(errors="replace"))
        if pr.returncode != 0:
            raise RuntimeError("nvcc failed: " + " ".join(cmd))
    tmp = LIB + ".tmp"
    cmd = [nvcc()] + ARCH + ["-shared", "-o", tmp] + objs + ["-lcudart"]
    subprocess.check_call(cmd)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
