"""Build recipe for the in-tree C-ABI library ``moss_image_b200/libmoss_w8.so``.

The library is plain CUDA C++ (no torch headers): nvcc compiles every ``csrc/*.cu`` for
sm_100a only and links them into one shared object with the CUDA runtime linked
statically, so the ``.so`` travels with the source tree and needs only the driver.

    python -m moss_image_b200.build          # incremental
    python -m moss_image_b200.build --force  # rebuild everything
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_DIR = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = PACKAGE_DIR / "_build"
LIB_PATH = PACKAGE_DIR / "libmoss_w8.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-v",
]


def nvcc_path() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the moss_image_b200 CUDA library cannot be built")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(dep.stat().st_mtime > t for dep in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link the library if any source is newer than the output."""
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(exist_ok=True)
    headers = _headers()
    objects = []
    for src in _sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *headers]):
            cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
            proc = subprocess.run(cmd, capture_output=True, text=True)
            log = BUILD_DIR / (src.stem + ".log")
            log.write_text(proc.stdout + proc.stderr)
            if proc.returncode != 0:
                sys.stderr.write(proc.stdout + proc.stderr)
                raise RuntimeError(f"nvcc failed on {src.name} (see {log})")
            if verbose:
                sys.stdout.write(proc.stderr)
    if force or _stale(LIB_PATH, objects):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            sys.stderr.write(proc.stdout + proc.stderr)
            raise RuntimeError("nvcc link of libmoss_w8.so failed")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    path = build(force=args.force, verbose=args.verbose)
    print(path)


if __name__ == "__main__":
    main()
