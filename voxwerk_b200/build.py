"""Build step for libvwsampler.so (sm_100a) and the test oracle.

``python -m voxwerk_b200.build`` compiles, in place:
  * voxwerk_b200/libvwsampler.so  -- nvcc -gencode arch=compute_100a,code=sm_100a (voxwerk_b200/csrc/Makefile)
  * oracle/liboracle.so           -- the CPU restatement used by tests and the benchmark's CPU baseline
"""

from __future__ import annotations

import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _make(directory: str) -> None:
    subprocess.run(["make", "-s", "-C", directory], check=True)


def build_library() -> str:
    _make(os.path.join(ROOT, "voxwerk_b200", "csrc"))
    return os.path.join(ROOT, "voxwerk_b200", "libvwsampler.so")


def build_oracle() -> str:
    _make(os.path.join(ROOT, "oracle"))
    return os.path.join(ROOT, "oracle", "liboracle.so")


def main() -> int:
    print(build_library())
    print(build_oracle())
    return 0


if __name__ == "__main__":
    sys.exit(main())
