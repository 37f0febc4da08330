"""Build librbt_moe.so for sm_100a (nvcc cross-compiles; no GPU needed)."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def build_library(jobs: int = 8) -> str:
    subprocess.run(["make", "-s", f"-j{jobs}", "-C", os.path.join(HERE, "csrc")], check=True)
    return os.path.join(HERE, "librbt_moe.so")


if __name__ == "__main__":
    print(build_library())
