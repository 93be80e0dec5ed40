"""Build ``libnqb.so`` (the C-ABI CUDA library) in-tree with nvcc for sm_100a.

Usage: ``python -m nanoquant_b200.build [--force] [--trace]``.  The library
lands in ``nanoquant_b200/_lib/libnqb.so``; sources are
``nanoquant_b200/csrc/*.cu``.  ``--trace`` builds the same sources with
``NQB_PHASE_TRACE`` into ``_lib/libnqb_trace.so``: the persistent decode
program then records per-stage cycle counts of its phases
(``nqb_program_trace``; see ``nanoquant_b200.program_trace``).  The build runs
without a GPU (nvcc cross-compiles).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
SOURCE_DIR = PACKAGE_DIR / "csrc"
LIB_DIR = PACKAGE_DIR / "_lib"
LIB_PATH = LIB_DIR / "libnqb.so"
TRACE_LIB_PATH = LIB_DIR / "libnqb_trace.so"
INCLUDE_DIR = PACKAGE_DIR.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3,-Wall",
    "-Xptxas",
    "-v",
]


def _nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    raise RuntimeError("nvcc not found; set CUDA_HOME")


def _sources() -> list[Path]:
    return sorted(SOURCE_DIR.glob("*.cu"))


def _inputs() -> list[Path]:
    return _sources() + sorted(SOURCE_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def is_stale(trace: bool = False) -> bool:
    path = TRACE_LIB_PATH if trace else LIB_PATH
    if not path.exists():
        return True
    built = path.stat().st_mtime
    return any(source.stat().st_mtime > built for source in _inputs())


def build(force: bool = False, verbose: bool = False, trace: bool = False) -> Path:
    """Compile every ``csrc/*.cu`` and link ``libnqb.so`` (or the trace build); returns its path."""

    target = TRACE_LIB_PATH if trace else LIB_PATH
    if not force and not is_stale(trace):
        return target
    nvcc = _nvcc()
    obj_dir = LIB_DIR / ("obj_trace" if trace else "obj")
    obj_dir.mkdir(parents=True, exist_ok=True)
    defines = ["-DNQB_PHASE_TRACE"] if trace else []
    headers = sorted(SOURCE_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))
    newest_header = max((h.stat().st_mtime for h in headers), default=0.0)

    def compile_one(source: Path) -> str:
        obj = obj_dir / (source.stem + ".o")
        if not force and obj.exists() and obj.stat().st_mtime > max(source.stat().st_mtime, newest_header):
            return str(obj)  # up to date (incremental rebuild)
        cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, *defines, "-I", str(INCLUDE_DIR), "-c", str(source), "-o", str(obj)]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"nvcc failed for {source.name}:\n{result.stdout}\n{result.stderr}")
        if verbose:
            sys.stderr.write(result.stderr)
        (obj_dir / (source.stem + ".ptxas.txt")).write_text(result.stderr)
        return str(obj)

    # the translation units are independent: compile them in parallel
    with ThreadPoolExecutor(max_workers=max(1, min(len(_sources()), os.cpu_count() or 1))) as pool:
        objects = list(pool.map(compile_one, _sources()))
    tmp = target.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *objects]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{result.stdout}\n{result.stderr}")
    os.replace(tmp, target)
    return target


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--trace", action="store_true", help="build the phase-trace variant libnqb_trace.so")
    args = parser.parse_args()
    path = build(force=args.force, verbose=args.verbose, trace=args.trace)
    print(path)


if __name__ == "__main__":
    main()
