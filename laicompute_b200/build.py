"""Build recipe of the native library (sm_100a CUDA + C++ host surface).

Outputs, in-tree:
  laicompute_b200/lib/liblaic_b200.so   C ABI (include/laic_b200.h) + C++ API (include/laic/*.hpp)
  laicompute_b200/bin/laic_generate     command-line generator (the reference's tools/generate usage)
  laicompute_b200/bin/laic_server       HTTP API server (the reference's tools/server usage)

Objects go to laicompute_b200/_build/ and are rebuilt only when a source or
header is newer than them.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "lib", "liblaic_b200.so")
BIN = os.path.join(PKG, "bin", "laic_generate")
INCLUDE = os.path.join(ROOT, "include")

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-std=c++17", "-O3", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC,-fvisibility=hidden", f"-I{INCLUDE}",
           f"-I{CSRC}"]
CXXFLAGS = ["-std=c++17", "-O2", "-fPIC", "-Wall", f"-I{INCLUDE}"]


def _cutlass_root() -> str:
    """CUTLASS/CuTe headers vendored in this image's Python packages (for the prefill GEMM)."""
    import sysconfig
    site = sysconfig.get_paths()["purelib"]
    for cand in (os.path.join(site, "flashinfer", "data", "cutlass"), os.path.join(site, "tilelang", "3rdparty", "cutlass")):
        if os.path.exists(os.path.join(cand, "include", "cute", "arch", "mma_sm100_umma.hpp")):
            return cand
    raise RuntimeError("CUTLASS headers with sm100 support not found")


def _nvflags(src: str) -> list:
    if os.path.basename(src) != "gemm_sm100.cu":
        return NVFLAGS
    root = _cutlass_root()
    return [*NVFLAGS, f"-I{root}/include", f"-I{root}/tools/util/include", "--expt-relaxed-constexpr"]


def _headers() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(INCLUDE, "**", "*.h*"), recursive=True))


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build failed: {' '.join(cmd[:3])} ...")


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    os.makedirs(os.path.dirname(BIN), exist_ok=True)
    hdrs = _headers()
    objs, jobs = [], []
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        if _stale(obj, [src, *hdrs]):
            jobs.append(("nvcc", src, [NVCC, *_nvflags(src), "-c", src, "-o", obj]))
        objs.append(obj)
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cpp"))):  # engine internals (not exported)
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        if _stale(obj, [src, *hdrs]):
            jobs.append(("g++", src, ["g++", *CXXFLAGS, "-fvisibility=hidden", "-c", src, "-o", obj]))
        objs.append(obj)
    for src in sorted(glob.glob(os.path.join(CSRC, "host", "*.cpp"))):
        obj = os.path.join(BUILD, "host_" + os.path.basename(src) + ".o")
        if _stale(obj, [src, *hdrs]):
            jobs.append(("g++", src, ["g++", *CXXFLAGS, "-c", src, "-o", obj]))
        objs.append(obj)
    for tool, src, _ in jobs:
        if verbose:
            print(tool, os.path.basename(src))
    with ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 1)) as ex:
        list(ex.map(lambda j: _run(j[2]), jobs))
    if _stale(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lpthread", "-ldl"])
    for tool in sorted(glob.glob(os.path.join(CSRC, "tools", "*.cpp"))):  # laic_generate, laic_server
        exe = os.path.join(os.path.dirname(BIN), os.path.splitext(os.path.basename(tool))[0])
        if _stale(exe, [tool, LIB, *hdrs]):
            _run(["g++", *CXXFLAGS, tool, "-o", exe, f"-L{os.path.dirname(LIB)}", "-llaic_b200",
                  "-Wl,-rpath,$ORIGIN/../lib", "-lpthread"])
    return LIB


if __name__ == "__main__":
    print(build(verbose=True))
