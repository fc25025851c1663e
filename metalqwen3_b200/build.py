"""Builds libq3cu.so in-tree with nvcc for sm_100a (see csrc/Makefile)."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")


def library_path() -> str:
    return os.path.join(HERE, "libq3cu.so")


def build_library(jobs: int | None = None, quiet: bool = True) -> str:
    """Compile (incrementally) every CUDA source into metalqwen3_b200/libq3cu.so."""
    jobs = jobs or max(1, min(8, os.cpu_count() or 1))
    cmd = ["make", "-C", CSRC, f"-j{jobs}"]
    if quiet:
        cmd.insert(1, "-s")
    subprocess.run(cmd, check=True)
    path = library_path()
    if not os.path.exists(path):
        raise RuntimeError(f"build finished but {path} is missing")
    return path
