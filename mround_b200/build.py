"""Compile ``libmround_b200.so`` for sm_100a with nvcc, in-tree.

``python -m mround_b200.build`` (or ``__graft_entry__.build()``) compiles every
``csrc/*.cu`` to an object and links them into ``mround_b200/libmround_b200.so``
next to this file.  Objects are rebuilt only when a source or header is newer.
There is no JIT path: the shared library is the product and travels with the
tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "libmround_b200.so"
INCLUDE = HERE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3",
    "-Xptxas",
    "-v" if os.environ.get("MR_PTXAS_VERBOSE") else "-O3",
]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cand = Path("/usr/local/cuda/bin/nvcc")
    if cand.exists():
        return str(cand)
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmround_b200.so")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _compile(src: Path, extra: list[str]) -> Path:
    obj = BUILD / (src.stem + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-I", str(CSRC), "-I", str(INCLUDE), "-c", str(src),
           "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if os.environ.get("MR_PTXAS_VERBOSE"):
        sys.stderr.write(res.stderr)
    return obj


def cutlass_include() -> list[str]:
    """CuTe/CUTLASS headers vendored with flashinfer (used as headers only)."""
    try:
        import importlib.util

        spec = importlib.util.find_spec("flashinfer")
        if spec and spec.origin:
            inc = Path(spec.origin).parent / "data" / "cutlass" / "include"
            if inc.exists():
                return ["-I", str(inc)]
    except Exception:  # pragma: no cover - optional header tree
        pass
    return []


def build(verbose: bool = False) -> Path:
    """Build (or refresh) the shared library and return its path."""
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    extra = cutlass_include()
    with ThreadPoolExecutor(max_workers=min(8, len(sources))) as pool:
        objs = list(pool.map(lambda s: _compile(s, extra), sources))
    if LIB.exists() and LIB.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
        return LIB
    cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(LIB)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build(verbose=True)
