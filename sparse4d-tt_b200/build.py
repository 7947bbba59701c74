"""Build ``lib/libs4d_dfa.so`` (the C ABI of ``include/s4d_dfa.h``) for sm_100a with nvcc.

    python sparse4d-tt_b200/build.py [--verbose-ptxas]

The library is built in-tree so that it travels with the repository; nothing is installed.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB_DIR = os.path.join(PKG, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libs4d_dfa.so")
SOURCES = ["capi.cu", "kps_project.cu", "dfa_gather.cu", "kps_noalloc.cu", "linear_tc.cu", "camera_encoder.cu", "pack_maps.cu",
           "instance_bank.cu", "peer.cu", "layer_norm.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def build(verbose_ptxas: bool = False, force: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith(".cuh")]
    deps.append(os.path.join(INCLUDE, "s4d_dfa.h"))
    if not force and os.path.exists(LIB_PATH):
        mt = os.path.getmtime(LIB_PATH)
        if all(os.path.getmtime(d) <= mt for d in deps) and not verbose_ptxas:
            return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "--shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "-I", INCLUDE, "-I", CSRC, "-o", LIB_PATH + ".tmp", *srcs,
           "-lcudart"]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libs4d_dfa.so")
    if verbose_ptxas:
        sys.stdout.write(res.stderr)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose_ptxas, a.force))
