"""In-tree build of megacu_b200's native libraries.

Everything is compiled with nvcc / g++ directly (no CMake, no JIT cache), so
the built ``.so`` files sit inside the repository and travel with it:

* ``megacu_b200/lib/libmegacu_b200.so`` — the C ABI (``include/megacu_b200.h``):
  host runtime (phase / dispatcher / ASAP scheduler), team (symmetric heap
  over CUDA IPC), and the sm_100a megakernels (``-gencode
  arch=compute_100a,code=sm_100a``).
* ``tests/_build/libhost_harness.so`` — the host-runtime test harness built
  against this repository's headers (test infrastructure).
* ``oracle/liboracle.so`` (+ ``oracle/_ref/*`` when the reference tree is
  present) via ``make -C oracle`` — the CPU checker (test infrastructure).
"""
from __future__ import annotations

import glob
import json
import os
import shutil
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "megacu_b200")
LIB_DIR = os.path.join(PKG, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libmegacu_b200.so")
# The same library with the kernels' bounds checks compiled in
# (-DMEGACU_B200_DEBUG_BOUNDS): loaded instead of the regular one when
# MEGACU_B200_LIBRARY=checked, for first runs of new kernel code.
CHECKED_LIB_PATH = os.path.join(LIB_DIR, "libmegacu_b200_checked.so")
HARNESS_PATH = os.path.join(ROOT, "tests", "_build", "libhost_harness.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + ["-lineinfo", "-O3", "-std=c++20", "-Xcompiler", "-fPIC",
                           "-Xcompiler", "-Wall"]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sm_100a kernels cannot be built")


def _sources() -> list[str]:
    src = sorted(glob.glob(os.path.join(PKG, "csrc", "*.cu")))
    src += sorted(glob.glob(os.path.join(PKG, "csrc", "runtime", "*.cc")))
    return src


def _deps() -> list[str]:
    deps = _sources()
    for pattern in ("csrc/**/*.h", "csrc/**/*.cuh"):
        deps += glob.glob(os.path.join(PKG, pattern), recursive=True)
    deps += glob.glob(os.path.join(ROOT, "include", "**", "*.h*"), recursive=True)
    return deps


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    proc = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def build_library(verbose: bool = False, force: bool = False, checked: bool = False) -> str:
    """Builds libmegacu_b200.so (or, with `checked`, the bounds-checked
    libmegacu_b200_checked.so) for sm_100a, skipped when up to date."""
    os.makedirs(LIB_DIR, exist_ok=True)
    path = CHECKED_LIB_PATH if checked else LIB_PATH
    if force or _stale(path, _deps()):
        tmp = path + ".tmp"
        cmd = [_nvcc(), *NVCC_FLAGS, *(["-DMEGACU_B200_DEBUG_BOUNDS"] if checked else []),
               "-shared", "-I" + os.path.join(ROOT, "include"),
               "-I" + os.path.join(PKG, "csrc"), *_sources(), "-o", tmp]
        _run(cmd, verbose)
        os.replace(tmp, path)
    return path


def build_harness(verbose: bool = False, force: bool = False) -> str:
    """Builds the host-runtime test harness against this repository's headers."""
    os.makedirs(os.path.dirname(HARNESS_PATH), exist_ok=True)
    src = [os.path.join(ROOT, "tests", "cpp", "host_runtime_harness.cc"),
           os.path.join(ROOT, "tests", "cpp", "co_resident_harness.cc")]
    src += sorted(glob.glob(os.path.join(PKG, "csrc", "runtime", "*.cc")))
    deps = src + glob.glob(os.path.join(ROOT, "include", "**", "*.h"), recursive=True)
    if force or _stale(HARNESS_PATH, deps):
        cxx = shutil.which("g++") or "g++"
        cmd = [cxx, "-O2", "-std=c++20", "-fPIC", "-shared", "-Wall",
               "-I" + os.path.join(ROOT, "include"), *src, "-o", HARNESS_PATH]
        _run(cmd, verbose)
    return HARNESS_PATH


def reference_root() -> str:
    """The reference tree named by BASELINE.json (reference_path), if present."""
    try:
        with open(os.path.join(ROOT, "BASELINE.json")) as f:
            path = json.load(f).get("reference_path") or ""
    except (OSError, ValueError):
        return ""
    return path if path and os.path.isdir(path) else ""


def build_oracle(verbose: bool = False) -> None:
    """Builds the CPU checker (and the reference builds when the tree exists)."""
    cmd = ["make", "-s", "-C", os.path.join(ROOT, "oracle")]
    ref = reference_root()
    if ref:
        cmd.append(f"REF={ref}")
    _run(cmd, verbose)


def kernel_resources() -> list[dict]:
    """ptxas' resource report of every kernel the library compiles (registers,
    spills, static shared memory), from `nvcc -Xptxas -v` of each source."""
    import re
    rows = []
    for src in sorted(glob.glob(os.path.join(PKG, "csrc", "*.cu"))):
        cmd = [_nvcc(), *NVCC_FLAGS, "-Xptxas", "-v", "-I" + os.path.join(ROOT, "include"),
               "-I" + os.path.join(PKG, "csrc"), "-c", src, "-o", os.devnull]
        proc = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(proc.stderr)
        name = None
        for line in proc.stderr.splitlines():
            m = re.search(r"Compiling entry function '([^']+)'", line)
            if m:
                name = m.group(1)
                rows.append({"source": os.path.basename(src), "kernel": name})
                continue
            m = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", line)
            if m and name and rows and rows[-1]["kernel"] == name:
                rows[-1]["spill_bytes"] = int(m.group(1)) + int(m.group(2))
            m = re.search(r"Used (\d+) registers", line)
            if m and name and rows and rows[-1]["kernel"] == name:
                rows[-1]["registers"] = int(m.group(1))
                sm = re.search(r"(\d+) bytes smem", line)
                rows[-1]["static_smem_bytes"] = int(sm.group(1)) if sm else 0
    return rows


def build_all(verbose: bool = False, force: bool = False) -> None:
    build_library(verbose, force)
    build_library(verbose, force, checked=True)
    build_harness(verbose, force)
    build_oracle(verbose)


if __name__ == "__main__":
    if "--resources" in sys.argv:
        for r in kernel_resources():
            print(f"{r['source']:12s} {r.get('registers', '?'):>4} regs "
                  f"{r.get('spill_bytes', 0):>4} B spill {r.get('static_smem_bytes', 0):>6} B smem "
                  f"{r['kernel']}")
    else:
        build_all(verbose=True, force="--force" in sys.argv)
