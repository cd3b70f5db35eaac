"""Builds libgfn_b200.so in-tree for sm_100a (nvcc; no GPU needed)."""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")


def build(verbose=False):
    """Run the csrc Makefile (incremental).  Raises on a compiler error."""
    res = subprocess.run(["make", "-j4", "-C", CSRC], capture_output=True, text=True)
    if verbose or res.returncode != 0:
        print(res.stdout)
        print(res.stderr)
    if res.returncode != 0:
        raise RuntimeError("building libgfn_b200.so failed")
    return os.path.join(HERE, "libgfn_b200.so")


if __name__ == "__main__":
    print(build(verbose=True))
