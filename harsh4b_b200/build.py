"""Build recipe for the sm_100a C-ABI library (libharsh4b_b200.so, in-tree)."""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
SOURCES = PACKAGE / "csrc"
LIBRARY = PACKAGE / "libharsh4b_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build harsh4b_b200")


def inputs() -> list[Path]:
    return sorted(SOURCES.glob("*.cu")) + sorted(SOURCES.glob("*.cuh")) + [
        PACKAGE.parent / "include" / "harsh4b_b200.h"]


def stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    return any(p.stat().st_mtime > built for p in inputs())


def build(force: bool = False, verbose: bool = False, output: Path | None = None,
          defines: tuple[str, ...] = ()) -> Path:
    """Compiles the library. `output`/`defines` make an instrumented copy
    elsewhere (e.g. defines=("H4B_PHASE_TRACE",) for the phase timeline)."""
    target = Path(output) if output is not None else LIBRARY
    if output is None and not force and not stale():
        return LIBRARY
    temporary = target.with_suffix(f".{os.getpid()}.tmp.so")
    command = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--shared", "-Xcompiler", "-fPIC",
               "-cudart", "static", f"-I{PACKAGE.parent / 'include'}", *(f"-D{d}" for d in defines),
               str(SOURCES / "harsh4b_b200.cu"), "-o", str(temporary)]
    if verbose:
        command.insert(1, "-Xptxas=-v")
    subprocess.run(command, check=True)
    os.replace(temporary, target)
    return target


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIBRARY)
