"""Generate the golden fixtures in this folder from the reference itself.

Run in a container that has the reference tree (the REF_ROOT environment
variable names it): it builds the reference's own CPU code from source into
oracle/_ref/ (oracle/build_oracle.py: recipe-lna/lna2/bindings.cpp with
orders/F1-ref/exl3_dequant.cuh) and records what that code returns on seeded
inputs.  The tests read only the .npz files written here, so they pin the
oracle on machines where the reference is absent.

Fixtures (all inputs are regenerated from the stored seeds by `inputs()`):
  ref_dequant.npz  dequant_trellis(trellis, suh, svh, K, mcg) of the reference
                   (bindings.cpp:118-133 -> dequant_cpu :16-101): full fp16
                   matrices for K in {2, 3} and sha256 digests for K in {4, 8},
                   mcg True (MCG) and False (MUL1)
  ref_codebook.npz sha256 of the reference's decode_codebook_bits over all
                   65536 windows for cb 0/1/2 (exl3_dequant.cuh:74-93), plus
                   its decode_mcg / decode_mul1 float values for 4096 windows
  ref_window.npz   read_window (exl3_dequant.cuh:110-128) at every weight start
                   of seeded tiles for K = 1..8
  ref_gemv.npz     the reference's CPU exl3_gemv (bindings.cpp:135-148:
                   dequant_cpu + at::mm in fp32, cast to x.dtype)
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

DEQUANT_CASES = [(K, mcg) for K in (2, 3, 4, 8) for mcg in (True, False)]
FULL_K = (2, 3)
GEMV_CASES = [(2, True, 1), (3, True, 2), (4, False, 3)]   # (K, mcg, rows)


def inputs(K: int, seed: int, kt: int = 8, nt: int = 8):
    """Seeded trellis / suh / svh in the EXL3 layout (numpy, platform independent)."""
    rng = np.random.default_rng(seed)
    trellis = rng.integers(-32768, 32768, size=(kt, nt, 16 * K), dtype=np.int16)
    suh = (1 - 2 * rng.integers(0, 2, kt * 16)).astype(np.float16)
    sv = 1 - 2 * rng.integers(0, 2, nt * 16)
    svh = (sv * np.abs(rng.standard_normal(nt * 16)) * 0.02).astype(np.float16)
    return trellis, suh, svh


def gemv_x(rows: int, k: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((rows, k)).astype(np.float16)


def case_seed(K: int, mcg: bool) -> int:
    return 1000 + 10 * K + int(mcg)


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> None:
    import torch

    from oracle import build_oracle as B
    from oracle import oracle as O

    B.build_all()
    ref = O.ref_ext()
    pin = O.ref_pin_lib()
    if ref is None or pin is None:
        raise SystemExit("the reference tree is needed to make the fixtures")

    out = {}
    for K, mcg in DEQUANT_CASES:
        t, su, sv = inputs(K, case_seed(K, mcg))
        w = ref.dequant_trellis(torch.from_numpy(t), torch.from_numpy(su), torch.from_numpy(sv), K, mcg).numpy()
        tag = f"K{K}_{'mcg' if mcg else 'mul1'}"
        out[f"sha_{tag}"] = np.array(digest(w.view(np.uint16)))
        if K in FULL_K:
            out[f"w_{tag}"] = w.view(np.uint16)
    np.savez_compressed(HERE / "ref_dequant.npz", **out)

    cbs = {}
    for cb in (0, 1, 2):
        table = np.array([pin.ref_decode_codebook_bits(w, cb) for w in range(65536)], dtype=np.uint16)
        cbs[f"sha_cb{cb}"] = np.array(digest(table))
    wins = np.arange(0, 65536, 16, dtype=np.uint16)
    cbs["windows"] = wins
    cbs["mcg_float"] = np.array([pin.ref_decode_mcg(int(w)) for w in wins], dtype=np.float32)
    cbs["mul1_float"] = np.array([pin.ref_decode_mul1(int(w)) for w in wins], dtype=np.float32)
    np.savez_compressed(HERE / "ref_codebook.npz", **cbs)

    wd = {}
    for K in range(1, 9):
        rng = np.random.default_rng(77 + K)
        tiles = rng.integers(0, 65536, size=(4, 16 * K), dtype=np.uint16)
        got = np.zeros((4, 256), dtype=np.uint16)
        for i in range(4):
            tile = np.ascontiguousarray(tiles[i])
            for t in range(256):
                got[i, t] = pin.ref_read_window(tile.ctypes.data, 16 * K, (t + 257) * K - 16)
        wd[f"tiles_K{K}"] = tiles
        wd[f"windows_K{K}"] = got
    np.savez_compressed(HERE / "ref_window.npz", **wd)

    gv = {}
    for K, mcg, rows in GEMV_CASES:
        t, su, sv = inputs(K, case_seed(K, mcg) + 500)
        x = gemv_x(rows, t.shape[0] * 16, 4000 + K)
        y = ref.exl3_gemv(torch.from_numpy(x), torch.from_numpy(t), torch.from_numpy(su), torch.from_numpy(sv),
                          K, mcg, 1).numpy()
        gv[f"y_K{K}_{int(mcg)}_{rows}"] = y.view(np.uint16)
    np.savez_compressed(HERE / "ref_gemv.npz", **gv)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
