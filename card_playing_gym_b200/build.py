"""Build the native library in-tree: card_playing_gym_b200/libcg_b200.so (sm_100a only).

    python -m card_playing_gym_b200.build [--force] [--verbose]

Every CUDA source under csrc/ is compiled with relocatable device code, then linked
(device link included) into one shared library that exports the C ABI declared in
include/cg_b200.h. No torch headers are involved: the library is plain CUDA C++.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
REPO = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = REPO / "include"
BUILD = PACKAGE / "_build"
LIBRARY = PACKAGE / "libcg_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC,-O3", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the native library needs the CUDA toolkit to build")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    stamp = target.stat().st_mtime
    return any(dep.stat().st_mtime > stamp for dep in deps)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    extra = list(extra or [])
    compiler = nvcc()
    jobs = []
    objects = []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *headers, Path(__file__)]):
            jobs.append([compiler, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)])

    def run(cmd: list[str]) -> None:
        if verbose:
            print(" ".join(cmd), flush=True)
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
        if verbose and (proc.stdout or proc.stderr):
            print(proc.stdout + proc.stderr, flush=True)

    workers = max(1, min(len(jobs), os.cpu_count() or 1))
    with concurrent.futures.ThreadPoolExecutor(workers) as pool:
        list(pool.map(run, jobs))
    if force or jobs or _stale(LIBRARY, objects):
        tmp = LIBRARY.with_suffix(".so.tmp")
        run([compiler, *ARCH, "-shared", "-rdc=true", *[str(o) for o in objects], "-o", str(tmp)])
        os.replace(tmp, LIBRARY)
    return LIBRARY


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    args = parser.parse_args(argv)
    extra = ["-Xptxas", "-v"] if args.ptxas_info else None
    path = build(force=args.force or args.ptxas_info, verbose=args.verbose or args.ptxas_info, extra=extra)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
