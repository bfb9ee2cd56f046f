"""Builds ``libasrback_attn.so`` (the C ABI of ``include/asrback_attn.h``) in-tree
with nvcc for sm_100a. Each ``csrc/*.cu`` compiles to an object in ``_build/``
only when it (or a header) changed; the objects link into ``_lib/``.

    python -m asrback_b200.build [--force] [--verbose]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
BUILD = PACKAGE / "_build"
LIB_DIR = PACKAGE / "_lib"
LIBRARY = LIB_DIR / "libasrback_attn.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    default = "/usr/local/cuda/bin/nvcc"
    if os.path.exists(default):
        return default
    raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build asrback_b200")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    stamp = target.stat().st_mtime
    return any(source.stat().st_mtime > stamp for source in sources)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compiles what changed and links the library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    compiler = nvcc()
    headers = _headers()
    sources = sorted(CSRC.glob("*.cu"))
    jobs = []
    objects = []
    for source in sources:
        obj = BUILD / (source.stem + ".o")
        objects.append(obj)
        if force or ptxas_info or _stale(obj, [source, *headers]):
            cmd = [compiler, *ARCH, *FLAGS, f"-I{INCLUDE}", "-c", str(source), "-o", str(obj)]
            if ptxas_info:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)

    def run(cmd: list[str]) -> subprocess.CompletedProcess:
        if verbose:
            print(" ".join(cmd), flush=True)
        return subprocess.run(cmd, capture_output=True, text=True)

    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as pool:
        for cmd, result in zip(jobs, pool.map(run, jobs)):
            if result.returncode != 0 or verbose or ptxas_info:
                sys.stderr.write(result.stdout + result.stderr)
            if result.returncode != 0:
                raise RuntimeError(f"nvcc failed for {cmd[-3]}")
    if jobs or force or _stale(LIBRARY, objects):
        cmd = [compiler, *ARCH, "-shared", "-o", str(LIBRARY), *map(str, objects), "-lcudart"]
        result = run(cmd)
        if result.returncode != 0:
            sys.stderr.write(result.stdout + result.stderr)
            raise RuntimeError("linking libasrback_attn.so failed")
    return LIBRARY


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true", help="rebuild every object")
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--ptxas-info", action="store_true", help="print registers/spills/smem")
    args = parser.parse_args()
    path = build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info)
    print(path)


if __name__ == "__main__":
    main()
