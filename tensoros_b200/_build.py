"""Build the native libraries in-tree.

Products (all under tensoros_b200/lib/, git-ignored, shipped with the tree):
  libtensoros_nn.so  sm_100a CUDA kernels + the C11 host runtime (C-ABI in
                     include/tensoros_nn_gpu.h)
  libtos_synth.so    seeded synthetic inputs (include/tos_synth.h), host C11

Every CUDA source is compiled with
  nvcc -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo -fmad=false
(-fmad=false keeps every fp32 rounding the reference performs: no FMA
contraction).  A content hash of sources and flags skips rebuilding when
nothing changed.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
INC = ROOT / "include"

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.environ.get("NVCC", str(Path(CUDA_HOME) / "bin" / "nvcc"))
CC = os.environ.get("CC", "gcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC",
                     "-I" + str(CSRC / "include"), "-I" + str(INC)]
CC_FLAGS = ["-std=c11", "-O2", "-fPIC", "-Wall", "-Wno-unused-function", "-D_GNU_SOURCE",
            "-I" + str(CSRC / "include"), "-I" + str(INC), "-I" + str(Path(CUDA_HOME) / "include")]

NN_CU = sorted((CSRC / "kernels").glob("*.cu"))
NN_C = [CSRC / "host" / "tos_runtime.c", CSRC / "host" / "tos_model.c", CSRC / "host" / "tos_shard.c",
        CSRC / "host" / "tos_gguf.c", CSRC / "host" / "tos_tf.c", CSRC / "host" / "tos_tensor.c"]
SYNTH_C = [CSRC / "host" / "tos_synth.c"]
HEADERS = (sorted((CSRC / "include").glob("*")) + sorted((CSRC / "kernels").glob("*.cuh"))
           + sorted(INC.glob("*.h")))

LIB_NN = LIB / "libtensoros_nn.so"
LIB_SYNTH = LIB / "libtos_synth.so"


def _hash(files, flags) -> str:
    h = hashlib.sha256()
    for f in files:
        h.update(str(f).encode())
        h.update(Path(f).read_bytes())
    h.update(" ".join(flags).encode())
    return h.hexdigest()


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), file=sys.stderr)
    subprocess.run([str(c) for c in cmd], check=True)


def _up_to_date(out: Path, digest: str) -> bool:
    stamp = out.with_suffix(out.suffix + ".hash")
    return out.exists() and stamp.exists() and stamp.read_text() == digest


def _stamp(out: Path, digest: str):
    out.with_suffix(out.suffix + ".hash").write_text(digest)


def build_synth(verbose=False) -> Path:
    LIB.mkdir(exist_ok=True)
    digest = _hash(SYNTH_C + HEADERS, CC_FLAGS)
    if _up_to_date(LIB_SYNTH, digest):
        return LIB_SYNTH
    _run([CC] + CC_FLAGS + ["-shared", "-o", LIB_SYNTH] + SYNTH_C + ["-lm", "-lpthread"], verbose)
    _stamp(LIB_SYNTH, digest)
    return LIB_SYNTH


def build_nn(verbose=False, jobs=None) -> Path:
    LIB.mkdir(exist_ok=True)
    digest = _hash(NN_CU + NN_C + HEADERS, NVCC_FLAGS + CC_FLAGS)
    if _up_to_date(LIB_NN, digest):
        return LIB_NN
    obj = ROOT / "_build" / "nn"
    obj.mkdir(parents=True, exist_ok=True)
    cmds = []
    objs = []
    for src in NN_CU:
        o = obj / (src.stem + ".o")
        objs.append(o)
        cmds.append([NVCC] + NVCC_FLAGS + ["-c", src, "-o", o])
    for src in NN_C:
        o = obj / (src.stem + ".o")
        objs.append(o)
        cmds.append([CC] + CC_FLAGS + ["-c", src, "-o", o])
    jobs = jobs or min(8, os.cpu_count() or 1)
    procs = []
    for c in cmds:
        if verbose:
            print(" ".join(str(x) for x in c), file=sys.stderr)
        procs.append(subprocess.Popen([str(x) for x in c]))
        if len(procs) >= jobs:
            if procs.pop(0).wait() != 0:
                raise RuntimeError("compile failed")
    for p in procs:
        if p.wait() != 0:
            raise RuntimeError("compile failed")
    tmp = LIB_NN.with_suffix(".so.tmp")
    _run([NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs + ["-lpthread", "-ldl"], verbose)
    os.replace(tmp, LIB_NN)
    _stamp(LIB_NN, digest)
    return LIB_NN


def build_oracle(verbose=False, with_reference=None):
    """Build the CPU checkers under oracle/ (test infrastructure).

    The reference's own sources are compiled (oracle/_ref) only when the
    environment variable TOS_REFERENCE_DIR names a TensorOS source tree."""
    ref_dir = os.environ.get("TOS_REFERENCE_DIR", "")
    ref = Path(ref_dir) if ref_dir else None
    targets = ["oracle"]
    if with_reference is None:
        with_reference = ref is not None and (ref / "runtime" / "nn" / "llm.c").exists()
    if with_reference:
        if ref is None:
            raise RuntimeError("TOS_REFERENCE_DIR must name the TensorOS source tree")
        targets.append("ref")
    make = shutil.which("make") or "make"
    _run([make, "-s", "-C", ROOT / "oracle"] + ([f"REF={ref}"] if ref else []) + targets, verbose)


def build_all(verbose=False):
    build_synth(verbose)
    build_nn(verbose)
    build_oracle(verbose)


if __name__ == "__main__":
    build_all(verbose="-v" in sys.argv)
