"""Build libnvfp4_moe_cuda.so (sm_100a) in-tree.

Every ``csrc/*.cu`` file is compiled by nvcc for ``sm_100a`` and linked into
``vllm_nvfp4_cuda/lib/libnvfp4_moe_cuda.so`` with the CUDA runtime linked
statically and only the ``nvfp4_*`` C symbols exported. Objects are rebuilt
when a source or header is newer than the library.

Usage: ``python x2-nvfp4-lab_b200/build.py [--force] [--verbose]``
"""

from __future__ import annotations

import argparse
import concurrent.futures as futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
LIB_DIR = HERE / "vllm_nvfp4_cuda" / "lib"
LIB = LIB_DIR / "libnvfp4_moe_cuda.so"
BUILD = HERE / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden,-O3",
    "-I",
    str(INCLUDE),
    "-I",
    str(CSRC),
]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    default = Path("/usr/local/cuda/bin/nvcc")
    if default.exists():
        return str(default)
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _compile(src: Path, obj: Path, verbose: bool) -> None:
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    if verbose and (proc.stdout or proc.stderr):
        sys.stderr.write(proc.stdout + proc.stderr)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link the library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    srcs = sources()
    newest_header = max((h.stat().st_mtime for h in headers()), default=0.0)
    lib_time = LIB.stat().st_mtime if LIB.exists() else -1.0
    jobs = []
    objs = []
    for src in srcs:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        stale = (
            force
            or not obj.exists()
            or obj.stat().st_mtime < src.stat().st_mtime
            or obj.stat().st_mtime < newest_header
        )
        if stale:
            jobs.append((src, obj))
    if jobs:
        workers = min(len(jobs), os.cpu_count() or 1)
        with futures.ThreadPoolExecutor(max_workers=workers) as pool:
            for fut in [pool.submit(_compile, s, o, verbose) for s, o in jobs]:
                fut.result()
    if jobs or lib_time < max(o.stat().st_mtime for o in objs):
        version_script = BUILD / "exports.map"
        version_script.write_text("{ global: nvfp4_*; local: *; };\n")
        cmd = [
            nvcc(),
            *ARCH_FLAGS,
            "-shared",
            "-cudart",
            "static",
            "-o",
            str(LIB),
            *map(str, objs),
            "-Xlinker",
            f"--version-script={version_script}",
            "-lrt",
            "-lpthread",
            "-ldl",
        ]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
    return LIB


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
