"""Compile libfastembedr_b200.so in-tree (sm_100a only).

    python -m fastembedr_b200.build_lib          # build if stale
    python -m fastembedr_b200.build_lib --force  # rebuild

nvcc cross-compiles without a GPU.  Flags of note:
  -gencode arch=compute_100a,code=sm_100a   B200 SASS, no PTX fallback
  --fmad=false   no multiply-add contraction, so float expressions round as
                 written (the reference CPU build is -O2 x86-64, which never
                 contracts); the kernels are bandwidth-bound, so this is free
  -lineinfo      source correlation for ncu
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libfastembedr_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

SOURCES = ["common.cu", "host_copy.cu", "nccl_loader.cu", "tsne_affinity.cu", "tsne_kernels.cu", "tsne_session.cu",
           "tsne_reorder.cu", "tsne_shard.cu", "multi_device.cu", "umap.cu", "umap_graph.cu", "umap_noalloc.cu", "umap_session.cu", "landmark.cu", "pca.cu", "knn.cu", "capi.cu"]
HEADERS = ["fe_common.cuh", "nccl_loader.cuh", "rank_group.h", "tsne.cuh", "umap.cuh"]

NVCC_FLAGS = [
    "-std=c++17", "-O3", "-lineinfo", "--fmad=false",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _inputs():
    files = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    files.append(os.path.join(INCLUDE, "fastembedr_b200.h"))
    files.append(os.path.abspath(__file__))
    return files


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(f) > t for f in _inputs())


def build(force: bool = False, verbose: bool = False, jobs: int = 0) -> str:
    if not force and not stale():
        return LIB
    objdir = os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    procs = []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        objs.append(obj)
        cmd = [NVCC, *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = False
    for src, p in procs:
        out, _ = p.communicate()
        text = out.decode(errors="replace")
        if p.returncode != 0:
            failed = True
            sys.stderr.write(f"--- nvcc failed on {src}\n{text}\n")
        elif verbose and text.strip():
            sys.stderr.write(f"--- {src}\n{text}\n")
    if failed:
        raise RuntimeError("nvcc compilation failed")
    # Export only the public C ABI: every extern "C" symbol is marked default
    # visibility by the header's linkage; internal C++ stays hidden.
    link = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-ldl", "-o", LIB + ".tmp"]
    subprocess.run(link, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
