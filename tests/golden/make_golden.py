"""Generate the golden GEMM fixtures in this folder from the CPU oracle.

    python tests/golden/make_golden.py

The reference repository holds no MLX output vectors for this path, so the fixtures are
oracle outputs on seeded inputs (fixed seeds, committed), plus the shapes the reference's
own self-test uses (``Worker/Sources/SmallMGEMM/SmallMGEMM.swift:251-279``).  They pin the
oracle against regressions (``tests/test_oracle_pins.py``) and give the GPU tests fixed
inputs (``tests/test_qgemm_gpu.py``).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import affine as A  # noqa: E402

# (name, m, n, k, bits, dtype, epilogue): K % 64 == 0 shapes of the reference self-test
# (GEMV rows 1-8, N not a multiple of the tile, K not a multiple of 256) and the native
# tile shapes (M 9-256).
CASES = [
    ("gemv_b4_m2_bias", 2, 96, 512, 4, "bf16", "bias"),
    ("gemv_b4_m4_res", 4, 136, 2048, 4, "bf16", "residual"),
    ("gemv_b8_m6_biasres", 6, 48, 128, 8, "bf16", "biasResidual"),
    ("gemv_b4_m7_gate", 7, 520, 1024, 4, "bf16", "siluGate"),
    ("gemv_b8_m1_none", 1, 136, 2048, 8, "bf16", "none"),
    ("gemv_d_m2_none", 2, 70, 3072, 0, "bf16", "none"),
    ("gemv_b4_f16_m5_bias", 5, 72, 768, 4, "f16", "bias"),
    ("gemv_d_f16_m8_gate", 8, 257, 640, 0, "f16", "siluGate"),
    ("tile_b4_m9_none", 9, 96, 320, 4, "bf16", "none"),
    ("tile_b8_m16_res", 16, 200, 1088, 8, "bf16", "residual"),
    ("tile_b4_m33_bias", 33, 64, 448, 4, "bf16", "bias"),
]


def make_case(seed: int, m: int, n: int, k: int, bits: int, dtype: str, epilogue: str) -> dict:
    rng = np.random.default_rng(seed)
    x = A.to_storage(rng.standard_normal((m, k)).astype(np.float32), dtype)
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    u = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    bias = A.to_storage(rng.standard_normal(n).astype(np.float32), dtype)
    res = A.to_storage(rng.standard_normal((m, n)).astype(np.float32), dtype)
    case = {"x": x, "bias": bias, "residual": res}
    if bits:
        case["w"], case["scales"], case["biases"] = A.quantize(w, bits, dtype)
        case["up_w"], case["up_scales"], case["up_biases"] = A.quantize(u, bits, dtype)
        up = (case["up_w"], case["up_scales"], case["up_biases"])
    else:
        case["w"] = A.to_storage(w, dtype)
        case["up_w"] = A.to_storage(u, dtype)
        up = (case["up_w"], None, None)
    case["out"] = A.qgemm(x, case["w"], case.get("scales"), case.get("biases"), bits=bits, dtype=dtype,
                          epilogue=epilogue, bias=bias, residual=res, up=up)
    if epilogue != "siluGate":
        for key in ("up_w", "up_scales", "up_biases"):
            case.pop(key, None)
    if epilogue not in ("bias", "biasResidual", "biasGelu", "biasGeluResidual"):
        case.pop("bias")
    if epilogue not in ("residual", "biasResidual", "biasGeluResidual"):
        case.pop("residual")
    case["meta"] = np.array([m, n, k, bits, 0 if dtype == "bf16" else 1, A.EPILOGUES.index(epilogue)], np.int64)
    return case


def main() -> None:
    arrays = {}
    for i, (name, *spec) in enumerate(CASES):
        for key, val in make_case(1000 + i, *spec).items():
            arrays[f"{name}/{key}"] = val
    path = os.path.join(HERE, "qgemm_cases.npz")
    np.savez_compressed(path, **arrays)
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
