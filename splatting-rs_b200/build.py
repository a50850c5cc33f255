"""Builds libsplat_b200.so in-tree (splat_b200/libsplat_b200.so) with nvcc for sm_100a.

Each CUDA source is compiled separately (in parallel) and linked into one shared library
with the CUDA runtime linked statically, so the library loads next to any other CUDA
runtime in the process (PyTorch's included). NCCL is not linked: comm.cu loads it at run
time (dlopen), so the library also loads where NCCL is absent. project.cu, adam.cu and densify.cu are
compiled with -fmad=false: their results are compared bit for bit with the CPU oracle; so
is pose_device.cu, so that its f64 pose chain rounds as the host's does.

    python splatting-rs_b200/build.py [--force] [--ptxas-verbose]
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
BUILD = HERE / "_build"
LIBRARY = HERE / "splat_b200" / "libsplat_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", f"-I{INCLUDE}", "--expt-relaxed-constexpr"]
EXACT = {"project.cu", "adam.cu", "pose_device.cu", "densify.cu"}
SOURCES = ["project.cu", "sort.cu", "blend.cu", "loss.cu", "adam.cu", "api.cu", "comm.cu", "pose.cpp",
           "pose_device.cu", "densify.cu", "noalloc.cu", "ply.cpp"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libsplat_b200")
    return path


def _headers() -> list[Path]:
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(source: str, ptxas_verbose: bool) -> tuple[str, str]:
    src = CSRC / source
    obj = BUILD / (source + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if source in EXACT:
        cmd.insert(1, "-fmad=false")
    if ptxas_verbose and source.endswith(".cu"):
        cmd += ["-Xptxas", "-v"]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed on {source}:\n{result.stderr}")
    return source, result.stderr


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = True) -> Path:
    """Compiles what changed and links the library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    headers = _headers()
    todo = [s for s in SOURCES if force or ptxas_verbose or _stale(BUILD / (s + ".o"), [CSRC / s, *headers])]
    reports = []
    if todo:
        with concurrent.futures.ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as pool:
            for source, err in pool.map(lambda s: _compile(s, ptxas_verbose), todo):
                if err.strip():
                    reports.append(f"== {source}\n{err}")
    objects = [BUILD / (s + ".o") for s in SOURCES]
    if todo or _stale(LIBRARY, objects):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIBRARY), *map(str, objects), "-ldl"]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"link failed:\n{result.stderr}")
    if reports and not quiet:
        print("\n".join(reports))
    return LIBRARY


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--ptxas-verbose", action="store_true")
    args = parser.parse_args()
    path = build(force=args.force, ptxas_verbose=args.ptxas_verbose, quiet=False)
    print(path)


if __name__ == "__main__":
    sys.exit(main())
