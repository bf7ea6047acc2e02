"""Build the C restatement of the lab's CPU path (test infrastructure only).

Compiles ``oracle/cpu_moe.c`` into ``oracle/_build/libnvfp4_cpu_oracle.so``
with gcc. ``-ffp-contract=off`` keeps every multiply and add separately
rounded, as the lab's non-fused NEON multiply-accumulate does; the target
is x86-64-v3 so the library runs on any AVX2 host.

The lab's own CPU GEMV (native_nvfp4/runtime/nvfp4_cpu.cpp) includes
<arm_neon.h> and cannot be compiled for this x86-64 host, so no build of the
reference itself exists here.
"""

from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "cpu_moe.c"
OUT_DIR = HERE / "_build"
LIB = OUT_DIR / "libnvfp4_cpu_oracle.so"


def build(force: bool = False) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    cmd = [
        "gcc",
        "-O3",
        "-march=x86-64-v3",
        "-ffp-contract=off",
        "-fPIC",
        "-shared",
        "-std=c11",
        str(SRC),
        "-o",
        str(LIB),
        "-lpthread",
        "-lm",
    ]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"gcc failed:\n{proc.stdout}\n{proc.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force=True))
