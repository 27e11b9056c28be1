"""Builds the sm_100a shared library libvoxcpm_b200.so in-tree with nvcc.

The library has a plain C ABI (include/voxcpm_b200.h) and links only the
CUDA runtime, so it loads into any process (ctypes here, cgo / JNI / dlopen
elsewhere). Usage: ``python -m voxcpm_b200.build [--force]``.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
LIBRARY = PACKAGE / "libvoxcpm_b200.so"
BUILD_DIR = ROOT / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-I",
    str(ROOT / "include"),
]


def _nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda) / "bin" / "nvcc"
    return str(candidate) if candidate.exists() else "nvcc"


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def _stale(target: Path, inputs: list[Path]) -> bool:
    if not target.exists():
        return True
    stamp = target.stat().st_mtime
    return any(p.stat().st_mtime > stamp for p in inputs)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles every source for sm_100a and links the shared library."""
    BUILD_DIR.mkdir(exist_ok=True)
    headers = (
        sorted(CSRC.glob("*.cuh"))
        + sorted(CSRC.glob("*.h"))
        + sorted((ROOT / "include").glob("*.h"))
    )
    objects = []
    jobs = []
    for source in sources():
        obj = BUILD_DIR / (source.name + ".o")
        objects.append(obj)
        if force or _stale(obj, [source] + headers):
            cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(source), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append((source, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for source, proc in jobs:
        out, _ = proc.communicate()
        text = out.decode(errors="replace")
        if proc.returncode != 0:
            failed.append(f"{source.name}:\n{text}")
        elif verbose and text:
            print(text)
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    if force or jobs or _stale(LIBRARY, objects):
        cmd = [
            _nvcc(),
            *ARCH_FLAGS,
            "-shared",
            "-o",
            str(LIBRARY),
            *map(str, objects),
            "-lcudart",
        ]
        subprocess.run(cmd, check=True)
    return LIBRARY


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIBRARY)
