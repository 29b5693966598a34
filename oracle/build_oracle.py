"""Build recipe for the CPU oracle and for the reference pins.

TEST INFRASTRUCTURE ONLY.  Produces
  oracle/_build/libexl3_oracle.so      the C restatement (always)
  oracle/_ref/libexl3_ref_pin.so       the reference's host decode helpers,
                                       compiled from orders/F1-ref/exl3_dequant.cuh
                                       where it lies in the reference tree
  oracle/_ref/vllm_exl3_c_ref*.so      the reference's recipe-lna/lna2/bindings.cpp
                                       built CPU-only as a torch extension
                                       (dequant_cpu + at::mm: the timed CPU baseline)
The two _ref builds need the reference tree (the REF_ROOT environment variable
names it) and are skipped when it is absent; the built files travel with the repository
snapshot, so nothing reads the reference tree at run time.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
REF_OUT = HERE / "_ref"
# The reference tree, named by the REF_ROOT environment variable; without it
# the _ref builds are skipped and any already built in oracle/_ref are used.
REF_ROOT = Path(os.environ["REF_ROOT"]) if os.environ.get("REF_ROOT") else None
ORACLE_SO = BUILD / "libexl3_oracle.so"
REF_PIN_SO = REF_OUT / "libexl3_ref_pin.so"
REF_EXT_NAME = "vllm_exl3_c_ref"


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def _stale(out: Path, srcs: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(s.stat().st_mtime > t for s in srcs)


def build_oracle(force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = [HERE / "exl3_oracle.c", HERE / "exl3_oracle.h"]
    if force or _stale(ORACLE_SO, srcs):
        _run(["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-std=c11", "-shared",
              "-fPIC", "-pthread", "-o", str(ORACLE_SO), str(HERE / "exl3_oracle.c"), "-lm"])
    return ORACLE_SO


def ref_available() -> bool:
    return REF_ROOT is not None and (REF_ROOT / "orders/F1-ref/exl3_dequant.cuh").is_file()


def ref_ext_path() -> Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return REF_OUT / f"{REF_EXT_NAME}{suffix}"


def build_ref_pin(force: bool = False) -> Path | None:
    if not ref_available():
        return REF_PIN_SO if REF_PIN_SO.exists() else None
    REF_OUT.mkdir(exist_ok=True)
    hdr = REF_ROOT / "orders/F1-ref/exl3_dequant.cuh"
    src = HERE / "ref_glue/ref_pin.cpp"
    if force or _stale(REF_PIN_SO, [hdr, src]):
        _run(["g++", "-O2", "-ffp-contract=off", "-std=c++17", "-shared", "-fPIC",
              "-I", str(REF_ROOT / "orders/F1-ref"), "-o", str(REF_PIN_SO), str(src)])
    return REF_PIN_SO


def build_ref_ext(force: bool = False) -> Path | None:
    """Compile the reference's bindings.cpp (CPU path) as module vllm_exl3_c_ref."""
    out = ref_ext_path()
    if not ref_available():
        return out if out.exists() else None
    import torch
    from torch.utils import cpp_extension

    REF_OUT.mkdir(exist_ok=True)
    bindings = REF_ROOT / "recipe-lna/lna2/bindings.cpp"
    glue = HERE / "ref_glue/gpu_entries_absent.cpp"
    srcs = [bindings, glue, REF_ROOT / "orders/F1-ref/exl3_dequant.cuh",
            HERE / "ref_glue/p2b_batched.cuh", HERE / "ref_glue/exl3_gemm.cuh"]
    if not (force or _stale(out, srcs)):
        return out
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O3", "-std=c++17", "-shared", "-fPIC", "-w",
           f"-DTORCH_EXTENSION_NAME={REF_EXT_NAME}", "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-I", str(HERE / "ref_glue"),
           "-I", str(REF_ROOT / "orders/F1-ref"),
           "-I", str(REF_ROOT / "recipe-lna/lna2"),
           "-I", sysconfig.get_paths()["include"]]
    for inc in cpp_extension.include_paths():
        cmd += ["-I", inc]
    cmd += [str(bindings), str(glue)]
    for lib in cpp_extension.library_paths():
        cmd += ["-L", lib, f"-Wl,-rpath,{lib}"]
    cmd += ["-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-o", str(out)]
    _run(cmd)
    return out


def build_all(force: bool = False) -> dict:
    res = {"oracle": str(build_oracle(force))}
    pin = build_ref_pin(force)
    res["ref_pin"] = str(pin) if pin else None
    ext = build_ref_ext(force)
    res["ref_ext"] = str(ext) if ext else None
    return res


if __name__ == "__main__":
    print(build_all(force="--force" in sys.argv))
