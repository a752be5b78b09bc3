"""Build oracle/_ref/libptcg_ref.so: the reference's own CUDA code for the
PPO loss, the rollout sampler and the negamax advantage, behind the C entry
points of oracle/ref_harness.cu.  TEST INFRASTRUCTURE ONLY: the pin tests
load it as a checker; nothing in the product path does.

The harness includes the reference's native/src/pufferlib.cu (which brings
models.cu, ocean.cu and native/model/*.cu) from the checkout named by
--ref or $PTCG_REFERENCE, with the reference trainer's own compile flags
(native/build_native.sh:80-88, fp32).  Nothing of the reference is copied
into this repository; the built library lands in oracle/_ref/, which git
ignores and which travels to the GPU box with the working tree.  The C env
(native/ptcg) is not linked: the harness calls none of it.

Usage: python oracle/build_ref.py --ref <reference checkout> [--force]
"""
import argparse
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT_DIR, "libptcg_ref.so")
SRC = os.path.join(HERE, "ref_harness.cu")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.environ.get("NVCC", os.path.join(CUDA, "bin", "nvcc"))


def _nccl():
    """(include dir, lib dir) of an NCCL install: the system one or the
    wheel torch ships with."""
    inc, lib = None, None
    for d in ("/usr/include", os.path.join(CUDA, "include")):
        if os.path.exists(os.path.join(d, "nccl.h")):
            inc = d
            break
    try:
        import nvidia.nccl as nn
        root = list(nn.__path__)[0]
        inc = inc or os.path.join(root, "include")
        if os.path.isdir(os.path.join(root, "lib")):
            lib = os.path.join(root, "lib")
    except (ImportError, IndexError):
        pass
    for d in ("/usr/lib/x86_64-linux-gnu", os.path.join(CUDA, "lib64")):
        if glob.glob(os.path.join(d, "libnccl.so*")):
            lib = lib or d
    return inc, lib


def build(ref, force=False, verbose=False):
    src_dir = os.path.join(ref, "native", "src")
    if not os.path.exists(os.path.join(src_dir, "pufferlib.cu")):
        raise FileNotFoundError(f"{src_dir}/pufferlib.cu not found: --ref must name a checkout "
                                "of the reference")
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) > os.path.getmtime(SRC):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    nv = os.path.join(ref, "native")
    inc, nlib = _nccl()
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O2",
           "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fopenmp",
           "-DOBS_TENSOR_T=FloatTensor", "-DENV_NAME=ptcg", "-DPTCG_NATIVE", "-DPRECISION_FLOAT",
           "-I" + os.path.join(nv, "src"), "-I" + os.path.join(nv, "model"),
           "-I" + os.path.join(nv, "ptcg"), "-I" + os.path.join(nv, "vendor")]
    if inc:
        cmd.append("-I" + inc)
    cmd += [SRC, "-o", LIB, "-L" + os.path.join(CUDA, "lib64"),
            ]
    if nlib:
        cmd += ["-L" + nlib, "-Xlinker", "-rpath=" + nlib]
        cmd.append("-l:libnccl.so.2" if os.path.exists(os.path.join(nlib, "libnccl.so.2"))
                   else "-lnccl")
    # NVML (called only by trainer code the harness never runs) stays unresolved:
    # the driver provides it on GPU machines, and lazy binding never asks for it
    cmd += ["-lcudart", "-lcublas", "-lcublasLt", "-lcurand", "-lgomp",
            "-lpthread"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"building {LIB} failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("PTCG_REFERENCE"))
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    if not a.ref:
        ap.error("--ref (or PTCG_REFERENCE) must name a checkout of the reference")
    print(build(a.ref, a.force, verbose=True))
    sys.exit(0)
