"""Builds libllmc_b200.so in-tree with nvcc for sm_100a (B200).

    python -m llmcompressorsharp_b200.build        # or build() from Python

The library is plain C ABI (include/llmc_b200.h) over CUDA kernels; no torch headers are
involved, so the build is one nvcc invocation that cross-compiles without a GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libllmc_b200.so")


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    deps.append(os.path.join(ROOT, "include", "llmc_b200.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def _flags() -> list[str]:
    return ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
            "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-I", os.path.join(ROOT, "include")]


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every .cu to an object in parallel, then link the shared library."""
    if not force and not _stale():
        return LIB
    from concurrent.futures import ThreadPoolExecutor

    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    nvcc = nvcc_path()

    def compile_one(src: str):
        obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc] + _flags() + (["-Xptxas=-v"] if verbose else []) + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, obj, r

    with ThreadPoolExecutor(max_workers=max(1, min(len(sources()), os.cpu_count() or 4))) as ex:
        results = list(ex.map(compile_one, sources()))
    failed = False
    for src, _, r in results:
        if r.returncode != 0 or verbose:
            sys.stderr.write(r.stdout + r.stderr)
        failed |= r.returncode != 0
    if failed:
        raise RuntimeError("nvcc build of libllmc_b200 failed")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC", "-o", LIB + ".tmp"]
    cmd += [obj for _, obj, _ in results]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("link of libllmc_b200 failed")
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
