"""Build recipe for the sm_100a paged-decode library (``libpaged_decode.so``).

The library is a plain shared object with the C ABI of ``include/paged_decode.h``; Python
binds it with ctypes (``model/_native.py``). Every translation unit is compiled with
``nvcc -gencode arch=compute_100a,code=sm_100a`` in parallel, then linked with the static
CUDA runtime, so the .so only needs the driver (``libcuda.so.1``) at run time and can be
loaded (not used) on a host without a GPU.

Usage: ``python llm-serving_b200/build.py [--force] [--verbose]``. The output lands next to
this file and is rebuilt only when a source is newer than it.
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
BUILD = HERE / "_build"
LIB = HERE / "libpaged_decode.so"

SOURCES = [
    "pd_api.cu",
    "pd_append.cu",
    "pd_merge.cu",
    "pd_decode_bf16.cu",
    "pd_decode_f16.cu",
    "pd_decode_f32.cu",
    "pd_decode_mma_bf16.cu",
    "pd_decode_mma_f16.cu",
    "pd_prefill.cu",
    "pd_prefill_tc.cu",
]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xptxas",
    "-O3",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]


def _nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cuda) / "bin" / "nvcc"
    return str(path) if path.exists() else "nvcc"


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(dep.stat().st_mtime > mtime for dep in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile and link the library; returns its path. Raises on a compiler error."""
    BUILD.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "paged_decode.h"]
    nvcc = _nvcc()
    objects = []
    jobs = []
    for name in SOURCES:
        src = CSRC / name
        obj = BUILD / (Path(name).stem + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *headers]):
            cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if ptxas_verbose:
                cmd[1:1] = ["-Xptxas", "-v"]
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        proc = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, proc

    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as pool:
        for cmd, proc in pool.map(run, jobs):
            if proc.returncode != 0 or verbose or ptxas_verbose:
                sys.stderr.write(proc.stdout + proc.stderr)
            if proc.returncode != 0:
                raise RuntimeError(f"nvcc failed ({proc.returncode}): {' '.join(cmd)}")

    if force or jobs or _stale(LIB, objects):
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objects)]
        if verbose:
            print(" ".join(cmd), flush=True)
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            sys.stderr.write(proc.stdout + proc.stderr)
            raise RuntimeError(f"link failed ({proc.returncode})")
    return LIB


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--ptxas-verbose", action="store_true", help="print registers/spills")
    args = parser.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas_verbose)
    print(path)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
