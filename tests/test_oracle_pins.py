"""Pins of the CPU oracle: the reference's own known answers for this path, restated.

No MLX outputs exist in the reference repository, so the oracle's GEMM is pinned by (a)
known-answer cases computed by hand from the layout the reference documents, (b) the
reference's dequant error bound, (c) the reference's self-test bound helpers, and (d) the
committed golden fixtures.
"""
import os

import numpy as np
import pytest

from oracle import affine as A

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "qgemm_cases.npz")


def test_pack_low_nibble_first():
    # SmallMGEMM.swift:491-493: 4-bit codes two per byte, low nibble first; element i of a
    # uint32 at bits [4i, 4i+4).  Codes 0..7 -> 0x76543210.
    codes = np.arange(8, dtype=np.uint8)[None, :]
    assert A.pack(codes, 4)[0, 0] == 0x76543210
    # 8-bit: element i at bits [8i, 8i+8) -> bytes in element order.
    assert A.pack(np.array([[1, 2, 3, 250]], np.uint8), 8)[0, 0] == 0xFA030201
    rng = np.random.default_rng(0)
    for bits in (4, 8):
        c = rng.integers(0, 1 << bits, size=(5, 128), dtype=np.uint8)
        assert np.array_equal(A.unpack(A.pack(c, bits), bits), c)


def test_known_answer_gemm_by_hand():
    # q[n][k] = (k + n) % 16, scale 0.5 / 0.25, bias -1 / 2, x = ones and x = k/64.
    k = np.arange(64)
    codes = np.stack([(k + n) % 16 for n in range(2)]).astype(np.uint8)
    packed = A.pack(codes, 4)
    scales = A.to_storage(np.array([[0.5], [0.25]], np.float32), "bf16")
    biases = A.to_storage(np.array([[-1.0], [2.0]], np.float32), "bf16")
    x = A.to_storage(np.stack([np.ones(64), k / 64.0]).astype(np.float32), "bf16")
    out = A.from_storage(A.qgemm(x, packed, scales, biases, bits=4), "bf16")
    # row 0: s * sum(q) + 64 b, sum(q) = 4 * (0 + ... + 15) = 480
    assert out[0, 0] == 0.5 * 480 - 64 and out[0, 1] == 0.25 * 480 + 128
    # row 1: sum_k (k/64) (s q + b), computed exactly
    exact = [sum((kk / 64.0) * (s * ((kk + n) % 16) + b) for kk in range(64))
             for n, (s, b) in enumerate([(0.5, -1.0), (0.25, 2.0)])]
    assert np.allclose(out[1], exact, rtol=2 ** -8)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_quantizer_within_reference_bound(bits, dtype):
    # NemotronTranscribeDerivationTests.swift:134-138 (affineBound), checked as :118-126 does.
    rng = np.random.default_rng(7)
    for scale in (0.02, 1.0):
        w = (rng.standard_normal((64, 1024)) * scale).astype(np.float32)
        p, s, b = A.quantize(w, bits, dtype)
        assert A.error_in_steps(w, p, s, b, bits, dtype) <= A.affine_bound(bits)
    # The edge of each group is exact in fp32 before the scale/bias are stored (zero stays zero).
    w = np.zeros((2, 64), np.float32)
    p, s, b = A.quantize(w, bits, dtype)
    assert np.all(A.dequantize(p, s, b, bits, dtype) == 0)


def test_affine_bound_values():
    assert A.affine_bound(4) == pytest.approx(0.5 + 1 + 2 * 15 / 256 + 0.05)
    assert A.affine_bound(8) == pytest.approx(0.5 + 1 + 2 * 255 / 256 + 0.05)


def test_self_test_bounds_and_failures():
    # GateTests.swift:533-541 (SmallM.revisionsAndBounds)
    assert A.self_test_bound("qtile.bf16.affine8.none") == 3e-2
    assert A.self_test_bound("tile.bf16.dense.none") == 2e-2
    assert A.self_test_failures({}) == []
    assert A.self_test_failures({"tile.bf16.dense.none": 0.03, "gemv.bf16.affine4.none": 0.029}) == ["tile.bf16.dense.none"]
    assert A.self_test_failures({"tile.bf16.dense.none": float("inf")}) == ["tile.bf16.dense.none"]
    assert A.relative_rms(np.array([np.nan]), np.array([1.0])) == float("inf")


def test_bf16_rounding_matches_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(3)
    a = (rng.standard_normal(10000) * 10.0 ** rng.integers(-5, 5, 10000)).astype(np.float32)
    ours = A.round_to(a, "bf16")
    theirs = torch.from_numpy(a).to(torch.bfloat16).float().numpy()
    assert np.array_equal(ours, theirs)


def test_golden_fixtures_reproduce():
    from tests.golden.make_golden import CASES, make_case
    data = np.load(GOLDEN)
    for i, (name, *spec) in enumerate(CASES):
        fresh = make_case(1000 + i, *spec)
        for key, val in fresh.items():
            assert np.array_equal(data[f"{name}/{key}"], val), (name, key)


def test_c_restatement_equals_the_numpy_oracle():
    """The oracle's C GEMM (used for model-sized checks and the CPU baseline) computes the same
    product form as the numpy oracle: int4 / int8 / dense, row counts 1 to 40 (several blocks
    of 16), within fp32 summation-order differences."""
    import numpy as np

    from oracle import affine as A
    rng = np.random.default_rng(17)
    for bits, m, n, k in [(4, 1, 96, 512), (4, 5, 130, 2048), (8, 17, 64, 1024), (4, 40, 33, 640), (0, 19, 70, 768)]:
        x = A.to_storage(rng.standard_normal((m, k)).astype(np.float32), "bf16")
        w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
        if bits:
            p, s, b = A.quantize(w, bits)
            ref = A.qgemm(x, p, s, b, bits=bits, raw=True)
            with A.c_accumulation():
                got = A.qgemm(x, p, s, b, bits=bits, raw=True)
            # the dequantize-then-multiply form: C equals numpy, and both stay within the
            # rounding of one bf16 weight of the product form
            ref_t = A.qgemm(x, p, s, b, bits=bits, raw=True, form="tile")
            with A.c_accumulation():
                got_t = A.qgemm(x, p, s, b, bits=bits, raw=True, form="tile")
            assert np.abs(got_t - ref_t).max() <= 1e-5 * max(1.0, np.abs(ref_t).max()), (bits, m, n, k)
            assert A.relative_rms(ref_t, ref) <= 1e-2
        else:
            wd = A.to_storage(w, "bf16")
            ref = A.qgemm(x, wd, bits=0, raw=True)
            with A.c_accumulation():
                got = A.qgemm(x, wd, bits=0, raw=True)
        assert got.shape == ref.shape == (m, n)
        assert np.abs(got - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max()), (bits, m, n, k)
