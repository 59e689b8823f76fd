"""Build recipe for the CPU oracle (test infrastructure only).

Compiles ``oracle/aie_oracle.c`` into ``oracle/libaie_oracle.so`` with
``-ffp-contract=off`` so that no multiply-add is fused.  That reproduces the
rounding of ai-cpu's x86 scalar F32x4 fallback (crates/ai-cpu/src/simd.rs:189-300).
The target ISA is the x86-64 baseline (SSE2, 4-lane vectors like F32x4), so the
same binary runs on any host this repository is copied to.

The reference itself (Rust) cannot be compiled here: no Rust toolchain is
installed, so there is no ``oracle/_ref`` build.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "aie_oracle.c")
LIB = os.path.join(HERE, "libaie_oracle.so")

CFLAGS = ["-O3", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
          "-fvisibility=hidden", "-pthread", "-Wall", "-Wno-unused-function"]


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = ["gcc", *CFLAGS, SRC, "-o", LIB + ".tmp", "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
