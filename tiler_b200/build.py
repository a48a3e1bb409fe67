"""Builds libtiler_cuda.so in-tree for sm_100a (nvcc cross-compiles without a
GPU).  ``python -m tiler_b200.build``."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libtiler_cuda.so")


def build(verbose: bool = False) -> str:
    """make -C csrc; the ptxas report (registers, spills, shared memory per
    kernel) goes to tiler_b200/_build/ptxas.log."""
    r = subprocess.run(["make", "-C", CSRC], capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("building libtiler_cuda.so failed")
    if verbose:
        sys.stdout.write(r.stdout)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True))
