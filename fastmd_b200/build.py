"""Build libfastmd_b200.so in the package directory (nvcc, sm_100a only).

``python -m fastmd_b200.build`` compiles every ``csrc/*.cu`` to an object in
``_build/`` and links them into ``fastmd_b200/libfastmd_b200.so`` with the CUDA
runtime linked statically. Objects are rebuilt when their source, a header
or this file is newer. nvcc cross-compiles without a GPU.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIBRARY = PACKAGE / "libfastmd_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "--expt-relaxed-constexpr", "-I", str(INCLUDE), "-I", str(CSRC)]
# Per-file flags: the integrator rounds every operation as NumPy does (no FMA contraction); the
# neighbour predicates and the segment-attention recurrences follow the reference's FP32 operation
# order (no contraction either).
EXTRA = {
    "nhc.cu": ["--fmad=false"],
    "neighbors.cu": ["--fmad=false"],
    "segment_attention.cu": ["--fmad=false"],
    "gather_add_silu.cu": ["--fmad=false"],
    "gated_ln.cu": ["--fmad=false"],
    "bond_graph.cu": ["--fmad=false"],
}


def _nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(cuda) / "bin" / "nvcc"
    return str(path) if path.exists() else "nvcc"


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(src.stat().st_mtime > mtime for src in sources)


def _compile(source: Path, verbose: bool) -> Path:
    obj = BUILD / (source.stem + ".o")
    deps = [source, Path(__file__), *INCLUDE.glob("*.h"), *CSRC.glob("*.cuh")]
    if _stale(obj, deps):
        cmd = [_nvcc(), *ARCH, *COMMON, *EXTRA.get(source.name, []), "-c", str(source), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return obj


def build(verbose: bool = False) -> Path:
    """Compile and link the library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    if not sources:
        raise RuntimeError(f"no CUDA sources in {CSRC}")
    with ThreadPoolExecutor(max_workers=min(8, len(sources))) as pool:
        objects = list(pool.map(lambda s: _compile(s, verbose), sources))
    if _stale(LIBRARY, objects):
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv[1:]))
