"""Build the C part of the oracle (test infrastructure only).

    python oracle/build_oracle.py

Compiles oracle/reuse_cache_oracle.c with gcc into
oracle/_build/libskv_oracle.so.  The product library never links it.
"""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "reuse_cache_oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libskv_oracle.so")


def build() -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = ["gcc", "-O2", "-std=c11", "-shared", "-fPIC", SRC, "-o", LIB]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build())
