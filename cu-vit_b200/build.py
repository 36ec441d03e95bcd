"""Builds libcuvit_b200.so in-tree with nvcc for sm_100a.

Every translation unit under csrc/ is compiled in parallel into _build/, then linked into
cuvit/_lib/libcuvit_b200.so with the CUDA runtime linked statically, so the library carries
no dependency on whichever libcudart another package in the process loaded.
"""

from __future__ import annotations

import concurrent.futures
import os
import pathlib
import shutil
import subprocess
import sys

PACKAGE_DIR = pathlib.Path(__file__).resolve().parent
REPO_DIR = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
LIB_DIR = PACKAGE_DIR / "cuvit" / "_lib"
# variant -> (object directory, library, extra nvcc flags). "timeline" is the diagnostic
# build whose forward-path kernels stamp a device timeline (csrc/timeline.cuh).
VARIANTS = {
    "default": (PACKAGE_DIR / "_build", LIB_DIR / "libcuvit_b200.so", []),
    "timeline": (PACKAGE_DIR / "_build_timeline", LIB_DIR / "libcuvit_b200_timeline.so",
                 ["-DCUVIT_TIMELINE"]),
}
BUILD_DIR, LIBRARY, _ = VARIANTS["default"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-std=c++17",
    "-O3",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    f"-I{REPO_DIR / 'include'}",
    f"-I{CSRC}",
]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = pathlib.Path("/usr/local/cuda/bin/nvcc")
    if candidate.exists():
        return str(candidate)
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build cuvit_b200")


def _compile(source: pathlib.Path, verbose: bool, variant: str = "default") -> pathlib.Path:
    build_dir, _, extra = VARIANTS[variant]
    obj = build_dir / (source.stem + ".o")
    deps = [source] + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.hpp"))
    deps.append(REPO_DIR / "include" / "cuvit_b200.h")
    if obj.exists() and all(obj.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return obj
    cmd = [nvcc(), *COMMON_FLAGS, *extra, *ARCH_FLAGS, "-c", str(source), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed on {source.name}:\n{result.stdout}\n{result.stderr}")
    if verbose and result.stderr:
        print(result.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, variant: str = "default") -> pathlib.Path:
    """Compiles csrc/*.cu and links the shared library of `variant`; returns its path."""
    build_dir, library, _ = VARIANTS[variant]
    build_dir.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    workers = max(1, min(len(sources), os.cpu_count() or 1))
    with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
        objects = list(pool.map(lambda s: _compile(s, verbose, variant), sources))
    newest = max(o.stat().st_mtime for o in objects)
    if library.exists() and library.stat().st_mtime >= newest:
        return library
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", str(library), *map(str, objects)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
    return library


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv,
                variant="timeline" if "--timeline" in sys.argv else "default"))
