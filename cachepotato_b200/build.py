"""Builds the CUDA library in-tree (cachepotato_b200/_build/libcpg_b200.so, sm_100a).

    python -m cachepotato_b200.build
"""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "_build", "libcpg_b200.so")


def build(jobs: int = 4) -> str:
    subprocess.run(["make", "-s", "-C", CSRC, f"-j{jobs}"], check=True)
    if not os.path.exists(LIB):
        raise RuntimeError(f"build produced no {LIB}")
    return LIB


if __name__ == "__main__":
    print(build())
