"""In-tree build of libhexir_b200.so, the sm_100a kernel CUBIN and the tools.

Runs `make` in hexir_b200/csrc (nvcc -gencode arch=compute_100a,code=sm_100a
for the kernels, g++/gcc for the host side).  Output stays in the source
tree (hexir_b200/lib, hexir_b200/bin) so it travels with the repository
snapshot to a GPU machine; nothing is installed elsewhere.
"""

from __future__ import annotations

import os
import subprocess

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")


def build(jobs: int = 8, verbose: bool = False) -> None:
    cmd = ["make", "-C", CSRC, f"-j{jobs}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        print(res.stdout[-4000:])
        print(res.stderr[-4000:])
    if res.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}")


if __name__ == "__main__":
    build(verbose=True)
