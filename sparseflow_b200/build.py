"""Build the sm_100a C-ABI library ``libsparseflow_b200.so`` in-tree.

The library is compiled straight from ``csrc/*.cu`` with nvcc (no torch
headers: the ABI in ``include/sparseflow_b200.h`` takes plain pointers), so
the same ``.so`` serves the Python package (through ctypes) and any other
host language.

    python -m sparseflow_b200.build [--force]
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_PATH = PKG_DIR / "libsparseflow_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found: set NVCC or put /usr/local/cuda/bin on PATH")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


BUILD_DIR = PKG_DIR / "_build"


def _run(cmd: list[str]) -> subprocess.CompletedProcess:
    return subprocess.run(cmd, capture_output=True, text=True)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every csrc/*.cu to an object (in parallel) and link the .so."""
    headers = sorted(CSRC.glob("*.cuh")) + [REPO_DIR / "include" / "sparseflow_b200.h"]
    deps = sources() + headers
    if not force and not _stale(LIB_PATH, deps):
        return LIB_PATH
    BUILD_DIR.mkdir(exist_ok=True)
    common = [_nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "--expt-relaxed-constexpr", f"-I{REPO_DIR / 'include'}"]
    if verbose:
        common.append("-Xptxas=-v")
    jobs = []
    for src in sources():
        obj = BUILD_DIR / (src.stem + ".o")
        if force or _stale(obj, [src] + headers):
            jobs.append(common + ["-c", str(src), "-o", str(obj)])
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 4))) as ex:
        results = list(ex.map(_run, jobs))
    for cmd, res in zip(jobs, results):
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed ({res.returncode}): {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        if verbose:
            print(res.stderr)
    objs = [str(BUILD_DIR / (s.stem + ".o")) for s in sources()]
    link = [_nvcc(), *ARCH_FLAGS, "-shared", "-o", str(LIB_PATH) + ".tmp", *objs, "-lcudart"]
    res = _run(link)
    if res.returncode != 0:
        raise RuntimeError(f"link failed: {res.stderr}")
    os.replace(str(LIB_PATH) + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB_PATH)
