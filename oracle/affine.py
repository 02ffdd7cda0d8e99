"""MLX-affine int4/int8 weights and the small-M dequant GEMM, restated on the CPU (numpy).

Test infrastructure only (see ``oracle/__init__.py``).

Layout (reference ``Worker/Sources/SmallMGEMM/SmallMGEMM.swift:491-498``, ``:658-661``):
  * weight W [N, K] is quantized in groups of ``GROUP = 64`` consecutive K elements;
  * element = scale[n, g] * q + bias[n, g], q in [0, 2**bits - 1];
  * codes are packed into uint32 words along K, ``32 // bits`` per word, element i of
    a word at bits ``[bits*i, bits*(i+1))`` (low nibble / low byte first);
  * packed weight is [N, K * bits / 32] uint32, scales and biases [N, K / 64] in the
    activation dtype (bf16 or fp16).

GEMM (reference ``SmallMGEMM.swift:662-755``, the ``smallm_gemv_affine`` kernel): the
product form ``acc += s * sum(x*q) + b * sum(x)`` per group, fp32 accumulation, then the
epilogue in fp32 in the order GATE (silu(a) * u), bias, residual, one rounding to the
activation dtype (``:745-753``).

Quantizer: MLX's affine quantize (third-party, ``mlx`` pinned through mlx-swift
``901941965d82e4a216d4d117231d847d194c563d``, reference ``Worker/Package.resolved``).
The published algorithm, restated: per group w_min/w_max, scale = max((max-min)/n_bins,
1e-7) signed toward the larger-magnitude edge, the edge snapped to an integer code so
that it is exact, codes = clip(round((w - bias) / scale), 0, n_bins) computed with the
fp32 scale and bias, then scale and bias stored in the activation dtype.  The reference
test ``NemotronTranscribeDerivationTests.swift:134-138`` bounds the resulting error at
``0.5 + 1 + 2 * (2**bits - 1) / 256 + 0.05`` steps; ``affine_bound`` restates it.
"""
from __future__ import annotations

import contextlib

import numpy as np

GROUP = 64


# ---------------------------------------------------------------------------------------
# dtype helpers (bf16 is emulated on fp32 bit patterns, round to nearest even)
# ---------------------------------------------------------------------------------------

def bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even; NaN stays NaN."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = 0x7FC0
    return rounded


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to(a: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 values to ``dtype`` ("bf16" | "f16" | "f32") and return them as fp32."""
    a = np.asarray(a, dtype=np.float32)
    if dtype == "bf16":
        return bf16_from_bits(bf16_bits(a))
    if dtype == "f16":
        return a.astype(np.float16).astype(np.float32)
    if dtype == "f32":
        return a
    raise ValueError(dtype)


def to_storage(a: np.ndarray, dtype: str) -> np.ndarray:
    """fp32 -> the raw storage array of ``dtype`` (uint16 bits for bf16, float16, float32)."""
    if dtype == "bf16":
        return bf16_bits(a)
    if dtype == "f16":
        return np.asarray(a, dtype=np.float32).astype(np.float16)
    if dtype == "f32":
        return np.asarray(a, dtype=np.float32)
    raise ValueError(dtype)


def from_storage(a: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16_from_bits(a)
    return np.asarray(a).astype(np.float32)


# ---------------------------------------------------------------------------------------
# packing
# ---------------------------------------------------------------------------------------

def pack(codes: np.ndarray, bits: int) -> np.ndarray:
    """codes [N, K] (ints in [0, 2**bits)) -> packed uint32 [N, K*bits/32], low bits first."""
    per = 32 // bits
    n, k = codes.shape
    assert k % per == 0
    c = codes.astype(np.uint32).reshape(n, k // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * bits)[None, None, :]
    return np.bitwise_or.reduce(c << shifts, axis=2).astype(np.uint32)


def unpack(packed: np.ndarray, bits: int) -> np.ndarray:
    """packed uint32 [N, K*bits/32] -> codes [N, K] (uint8)."""
    per = 32 // bits
    mask = np.uint32((1 << bits) - 1)
    shifts = (np.arange(per, dtype=np.uint32) * bits)[None, None, :]
    codes = (packed[:, :, None] >> shifts) & mask
    return codes.reshape(packed.shape[0], -1).astype(np.uint8)


# ---------------------------------------------------------------------------------------
# quantize / dequantize
# ---------------------------------------------------------------------------------------

def _round_half_away(a: np.ndarray) -> np.ndarray:
    return np.sign(a) * np.floor(np.abs(a) + np.float32(0.5))


def quantize(w: np.ndarray, bits: int, dtype: str = "bf16", group: int = GROUP):
    """MLX affine quantize of w [N, K] (fp32) -> (packed uint32, scales, biases).

    scales/biases are returned in storage form of ``dtype`` (uint16 bf16 bits or float16).
    """
    assert bits in (4, 8) and group == GROUP
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    assert k % group == 0
    wg = w.reshape(n, k // group, group)
    n_bins = np.float32((1 << bits) - 1)
    eps = np.float32(1e-7)
    w_max = wg.max(axis=2)
    w_min = wg.min(axis=2)
    side = np.abs(w_min) > np.abs(w_max)
    scale = np.maximum((w_max - w_min) / n_bins, eps).astype(np.float32)
    scale = np.where(side, scale, -scale).astype(np.float32)
    edge = np.where(side, w_min, w_max).astype(np.float32)
    q0 = _round_half_away(edge / scale).astype(np.float32)
    at_zero = q0 == 0
    with np.errstate(divide="ignore", invalid="ignore"):
        snapped = (edge / np.where(at_zero, np.float32(1), q0)).astype(np.float32)
    scale = np.where(at_zero, scale, snapped).astype(np.float32)
    bias = np.where(at_zero, np.float32(0), edge).astype(np.float32)
    codes = _round_half_away((wg - bias[:, :, None]) / scale[:, :, None])
    codes = np.clip(codes, 0, n_bins).astype(np.uint32).reshape(n, k)
    return pack(codes, bits), to_storage(scale, dtype), to_storage(bias, dtype)


def dequantize(packed, scales, biases, bits: int, dtype: str = "bf16") -> np.ndarray:
    """Exact fp32 dequantization (s * q + b in fp32, not rounded)."""
    q = unpack(packed, bits).astype(np.float32)
    n, k = q.shape
    s = from_storage(scales, dtype)
    b = from_storage(biases, dtype)
    return (q.reshape(n, k // GROUP, GROUP) * s[:, :, None] + b[:, :, None]).reshape(n, k)


def affine_bound(bits: int) -> float:
    """Largest |source - dequantized| in steps of the group's stored scale (reference
    ``Worker/Tests/VellaWorkerTests/NemotronTranscribeDerivationTests.swift:134-138``)."""
    return 0.5 + 1 + 2 * float((1 << bits) - 1) / 256 + 0.05


def error_in_steps(source, packed, scales, biases, bits: int, dtype: str = "bf16") -> float:
    """Reference ``NemotronTranscribeDerivationTests.swift:118-126``: max error / |scale|."""
    deq = dequantize(packed, scales, biases, bits, dtype)
    n, k = deq.shape
    s = np.maximum(np.abs(from_storage(scales, dtype)), 1e-12)
    err = np.abs(np.asarray(source, np.float32) - deq).reshape(n, k // GROUP, GROUP)
    return float((err / s[:, :, None]).max())


# ---------------------------------------------------------------------------------------
# the GEMM
# ---------------------------------------------------------------------------------------

EPILOGUES = ("none", "bias", "residual", "biasResidual", "siluGate", "biasGelu", "biasGeluResidual")


_ENGINE = ["numpy"]


@contextlib.contextmanager
def c_accumulation(reverse: bool = False):
    """Inside the block, bf16 GEMM accumulations run in the C restatement of the same forms
    (``oracle/c/oracle_gemm.c``, OpenMP over output rows), for model-sized shapes where numpy
    takes minutes; fp16 ones stay in numpy.  ``reverse`` sums along K in descending order: the
    same arithmetic in another valid order, to measure how far rounding order alone moves a
    result."""
    from . import cgemm
    _ENGINE.append("c")
    cgemm.set_reverse(reverse)
    try:
        yield
    finally:
        cgemm.set_reverse(False)
        _ENGINE.pop()


def _affine_acc(x32: np.ndarray, packed, scales, biases, bits: int, dtype: str, chunk: int = 4096):
    """fp32 accumulators [M, N] in product form: sum_g s*sum(x*q) + b*sum(x)."""
    if _ENGINE[-1] == "c" and dtype == "bf16":
        from . import cgemm
        return cgemm.qgemm(x32, packed, scales, biases, bits)
    m, k = x32.shape
    g = k // GROUP
    xg = x32.reshape(m, g, GROUP)
    xs = xg.sum(axis=2)  # [M, G]
    s = from_storage(scales, dtype)
    b = from_storage(biases, dtype)
    n = packed.shape[0]
    out = np.empty((m, n), dtype=np.float32)
    for n0 in range(0, n, chunk):
        n1 = min(n, n0 + chunk)
        q = unpack(packed[n0:n1], bits).astype(np.float32).reshape(n1 - n0, g, GROUP)
        p = np.einsum("mgk,ngk->mng", xg, q, optimize=True)  # [M, n, G]
        acc = p * s[None, n0:n1, :] + xs[:, None, :] * b[None, n0:n1, :]
        out[:, n0:n1] = acc.sum(axis=2, dtype=np.float32)
    return out


def _dequant_acc(x32: np.ndarray, packed, scales, biases, bits: int, dtype: str, chunk: int = 4096):
    """fp32 accumulators [M, N] of the dequantize-then-multiply form: every weight is first
    rounded once to the activation dtype, W' = T(s * q + b), then sum_k x * W'.  This is the
    form of quantized matmuls that stage dequantized weight tiles for a matrix unit (stock
    MLX quantizedMM at large row counts, and the library's tensor-core GEMM for calls above 16
    rows); the GEMV form above keeps s and b outside the sum."""
    if _ENGINE[-1] == "c" and dtype == "bf16":
        from . import cgemm
        return cgemm.qgemm_tile(x32, packed, scales, biases, bits)
    m, k = x32.shape
    g = k // GROUP
    s = from_storage(scales, dtype).astype(np.float64)
    b = from_storage(biases, dtype).astype(np.float64)
    n = packed.shape[0]
    out = np.empty((m, n), dtype=np.float32)
    for n0 in range(0, n, chunk):
        n1 = min(n, n0 + chunk)
        q = unpack(packed[n0:n1], bits).astype(np.float64).reshape(n1 - n0, g, GROUP)
        w = q * s[n0:n1, :, None] + b[n0:n1, :, None]
        w = round_to(w.astype(np.float32).reshape(n1 - n0, k), dtype)
        out[:, n0:n1] = x32 @ w.T
    return out


def _dense_acc(x32: np.ndarray, w, dtype: str) -> np.ndarray:
    if _ENGINE[-1] == "c" and dtype == "bf16":
        from . import cgemm
        return cgemm.gemm_dense(x32, w)
    return x32 @ from_storage(w, dtype).T


def gelu(a: np.ndarray) -> np.ndarray:
    """GELU, erf form (MLX's default ``gelu``, used by the Whisper MLP and convolutions)."""
    from scipy.special import erf
    a = np.asarray(a, np.float32)
    return (0.5 * a * (1.0 + erf(a / np.float32(np.sqrt(2.0))).astype(np.float32))).astype(np.float32)


def silu(a: np.ndarray) -> np.ndarray:
    return a / (np.float32(1) + np.exp(-a))


def qgemm(x, w, scales=None, biases=None, *, bits: int = 4, dtype: str = "bf16",
          epilogue: str = "none", bias=None, residual=None, up=None, raw: bool = False, form: str = "product"):
    """out[M, N] = epilogue(x[M, K] . W^T) in the reference's order, rounded once.

    ``x``/``bias``/``residual`` are storage arrays of ``dtype``.  ``bits`` = 0 means dense
    W (storage of ``dtype``, [N, K]); otherwise ``w`` is the packed uint32 array with
    ``scales``/``biases``.  ``up`` = (w, scales, biases) of the up projection for
    ``siluGate``.  ``raw`` returns the fp32 result before the final rounding.  ``form``
    selects the quantized accumulation: "product" (the GEMV's s * sum(x q) + b * sum(x)) or
    "tile" (weights dequantized to the activation dtype first).
    """
    x32 = from_storage(x, dtype)

    def acc(wt, sc, bi):
        if bits == 0:
            return _dense_acc(x32, wt, dtype)
        if form == "tile":
            return _dequant_acc(x32, wt, sc, bi, bits, dtype)
        return _affine_acc(x32, wt, sc, bi, bits, dtype)

    a = acc(w, scales, biases)
    if epilogue == "siluGate":
        u = acc(*up)
        a = silu(a) * u
    if epilogue in ("bias", "biasResidual", "biasGelu", "biasGeluResidual"):
        a = a + from_storage(bias, dtype)[None, :]
    if epilogue in ("biasGelu", "biasGeluResidual"):
        a = gelu(a)
    if epilogue in ("residual", "biasResidual", "biasGeluResidual"):
        a = a + from_storage(residual, dtype)
    a = a.astype(np.float32)
    return a if raw else to_storage(a, dtype)


def relative_rms(a: np.ndarray, b: np.ndarray) -> float:
    """||a - b|| / ||b|| in fp32; inf when non-finite (reference ``SmallMGEMM.swift:379-383``)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    v = np.sqrt(((a - b) ** 2).sum() / (b ** 2).sum())
    return float(v) if np.isfinite(v) else float("inf")


def self_test_bound(class_name: str) -> float:
    """Self-test bound per weight format (reference ``SmallMGEMM.swift:369-371``)."""
    return 3e-2 if (".affine" in class_name or ".mxfp" in class_name) else 2e-2


def self_test_failures(results: dict) -> list:
    """Classes whose value is non-finite or above the bound (reference ``SmallMGEMM.swift:374-376``)."""
    return sorted(k for k, v in results.items() if not (v <= self_test_bound(k)))
