"""Build the C-ABI library dsv4_carve_b200/libexl3b200.so for sm_100a.

Plain nvcc: every csrc/*.cu is compiled to an object in _build/ (in parallel),
then linked into one shared library next to this file.  No torch headers are
involved: the library is the drop-in boundary, torch is only used by the
Python host layer for memory and streams.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG.parent / "_build" / "csrc"
LIB = PKG / "libexl3b200.so"
# Instrumented variant (-DEXL3_PHASE_CLOCK: per-phase clock64 accumulators in
# the MoE kernel, read with exl3_phase_clock_read); load it by pointing
# EXL3_B200_LIB at it.  Not used by the product path.
TRACE_BUILD = PKG.parent / "_build" / "csrc_trace"
TRACE_LIB = PKG / "libexl3b200_trace.so"
NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-I", str(PKG.parent / "include")]


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.hpp"))
                  + list((PKG.parent / "include").glob("*.h")))


def _compile(src: Path, verbose: bool, build_dir: Path = BUILD, extra: tuple = ()) -> Path:
    obj = build_dir / (src.stem + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stderr}")
    if verbose:
        sys.stderr.write(proc.stderr)
    return obj


def build(verbose: bool = False, force: bool = False, trace: bool = False) -> Path:
    build_dir, lib, extra = (TRACE_BUILD, TRACE_LIB, ("-DEXL3_PHASE_CLOCK",)) if trace else (BUILD, LIB, ())
    build_dir.mkdir(parents=True, exist_ok=True)
    srcs = _sources()
    if force:
        for o in build_dir.glob("*.o"):
            o.unlink()
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, build_dir, extra), srcs))
    if force or not lib.exists() or any(o.stat().st_mtime > lib.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(lib), *map(str, objs), "-cudart", "static"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stderr}")
    return lib


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="--force" in sys.argv, trace="--trace" in sys.argv))
