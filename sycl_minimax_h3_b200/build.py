"""Builds the product libraries in-tree (csrc/Makefile -> lib/libh3cuda.so, lib/libh3sage.so) for sm_100a."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def build(verbose: bool = False) -> None:
    cmd = ["make", "-C", os.path.join(HERE, "csrc")]
    if not verbose:
        cmd.insert(1, "-s")
    subprocess.run(cmd, check=True)


if __name__ == "__main__":
    build(verbose=True)
