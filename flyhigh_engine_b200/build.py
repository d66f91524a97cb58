"""Build recipe of the package's native code: libflyhigh.so (CUDA, sm_100a) from csrc/ with its Makefile."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def build(jobs: int = 3) -> str:
    """Compiles csrc/*.cu for sm_100a (nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo) into libflyhigh.so."""
    subprocess.run(["make", "-s", f"-j{jobs}", "-C", os.path.join(HERE, "csrc")], check=True)
    return os.path.join(HERE, "libflyhigh.so")


if __name__ == "__main__":
    print(build())
