"""Builds the C-ABI shared library ``lib/libpaged_serve_b200.so`` from ``csrc/*.cu``.

Plain ``nvcc`` (no torch headers, no JIT cache): every kernel is compiled for
``sm_100a`` only and linked with the static CUDA runtime, so the library depends
on nothing but the driver. Objects go to ``_build/`` beside this file and are
rebuilt only when a source or header is newer than its object.

Usage: ``python -m paged_serve_b200.build [--force] [--jobs N]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB_DIR = PKG / "lib"
LIB_NAME = "libpaged_serve_b200.so"
LIB_PATH = LIB_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    default = "/usr/local/cuda/bin/nvcc"
    if os.path.exists(default):
        return default
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build paged_serve_b200")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(
        (ROOT / "include").glob("*.h")
    )


def _stale(obj: Path, src: Path, headers: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *headers])


def _compile(nvcc: str, src: Path, obj: Path, extra: list[str]) -> tuple[Path, str]:
    cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    """Compile every ``csrc/*.cu`` and link the shared library; returns its path."""
    nvcc = nvcc_path()
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    headers = _headers()
    sources = sorted(CSRC.glob("*.cu"))
    extra = ["-Xptxas", "-v"] if verbose else []
    todo = []
    objs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, src, headers):
            todo.append((src, obj))
    if todo:
        jobs = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=jobs) as pool:
            futs = [pool.submit(_compile, nvcc, s, o, extra) for s, o in todo]
            for f in futs:
                _, log = f.result()
                if verbose and log:
                    print(log)
    if force or todo or not LIB_PATH.exists() or any(
        o.stat().st_mtime > LIB_PATH.stat().st_mtime for o in objs
    ):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    args = ap.parse_args()
    path = build(force=args.force, jobs=args.jobs, verbose=args.verbose)
    print(path)


if __name__ == "__main__":
    main()
