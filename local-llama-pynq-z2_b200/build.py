"""Builds libmatvec_b200.so in this directory from csrc/ with nvcc for sm_100a (no GPU needed).

usage: python build.py [--verbose]     (--verbose adds -Xptxas -v: registers, spills, shared memory per kernel)

-fmad=false: the reference's float arithmetic has no fused multiply-adds (its C is built with
-ffp-contract=off), so neither does any kernel here. The CUDA runtime is linked statically so that hosts built
from the reference's C (-lmatvec_b200) need nothing else.
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libmatvec_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC,-O2", "-shared", "-cudart", "static",
         "--expt-relaxed-constexpr"]


def sources():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")))


def up_to_date():
    if not os.path.exists(LIB):
        return False
    deps = sources() + glob.glob(os.path.join(HERE, "csrc", "*.cuh")) + glob.glob(os.path.join(HERE, "csrc", "*.h"))
    deps += glob.glob(os.path.join(HERE, "..", "include", "*.h")) + [os.path.abspath(__file__)]
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in deps)


def build(verbose=False, force=False):
    if not force and not verbose and up_to_date():
        return LIB
    cmd = [NVCC, *ARCH, *FLAGS, *(["-Xptxas", "-v"] if verbose else []), "-o", LIB + ".tmp", *sources()]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    if verbose:
        sys.stdout.write(r.stdout + r.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force=True))
