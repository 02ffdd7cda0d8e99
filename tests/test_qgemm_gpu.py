"""Parity of the CUDA small-M GEMM (vella_qgemm through the C ABI) with the CPU oracle.

Tolerance: relative RMS <= 1e-2 and max |error| <= 1e-2 * max |oracle| per call (the GEMM
bar of the decode path; the reference's own self-test allows 3e-2 affine / 2e-2 dense,
``SmallMGEMM.swift:369-371``).  Integer properties are exact: a row of a batched call is
bit-identical to the same row computed alone, and writes stay inside the output.
"""
import os

import numpy as np
import pytest
import torch

from oracle import affine as A
from tests._util import TORCH_DT, as_f32, dev, host

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "qgemm_cases.npz")
REL = 1e-2


def smallm():
    from vella_b200 import smallm as S
    return S


def weights(case, prefix, bits):
    S = smallm()
    if bits:
        return S.Weights(dev(case[f"{prefix}w"]), dev(case[f"{prefix}scales"]), dev(case[f"{prefix}biases"]), bits)
    return S.Weights(dev(case[f"{prefix}w"]), bits=0)


def assert_close(out, ref, dtype):
    o = as_f32(out, dtype).astype(np.float64)
    r = as_f32(ref, dtype).astype(np.float64)
    assert np.isfinite(o).all()
    rel = A.relative_rms(o, r)
    assert rel <= REL, rel
    assert np.abs(o - r).max() <= REL * max(np.abs(r).max(), 1e-6)


def run_case(case, m, n, k, bits, dtype, epi, rows=None):
    S = smallm()
    tdt = TORCH_DT[dtype]
    x = dev(case["x"], dtype)
    w = weights(case, "", bits)
    up = weights(case, "up_", bits) if epi == "siluGate" else None
    bias = dev(case["bias"], dtype) if "bias" in case else None
    res = dev(case["residual"], dtype) if "residual" in case else None
    out = S.matmul(x, w, epilogue=epi, bias=bias, residual=res, up=up)
    assert out is not None and out.dtype == tdt and tuple(out.shape) == (m, n)
    torch.cuda.synchronize()
    return host(out)


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_golden_fixtures(golden):
    from tests.golden.make_golden import CASES
    for name, m, n, k, bits, dtype, epi in CASES:
        case = {key.split("/", 1)[1]: golden[key] for key in golden.files if key.startswith(name + "/")}
        out = run_case(case, m, n, k, bits, dtype, epi)
        assert_close(out, case["out"], dtype)


def make(m, n, k, bits, dtype, epi, seed=0, scale=0.02):
    from tests.golden.make_golden import make_case
    return make_case(seed, m, n, k, bits, dtype, epi)


@pytest.mark.parametrize("bits", [0, 4, 8])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("epi", ["none", "bias", "residual", "biasResidual", "siluGate", "biasGelu",
                                 "biasGeluResidual"])
def test_every_class(bits, dtype, epi):
    # every row count 1..16, N not a multiple of the CTA tile, K not a multiple of 256
    for m, n, k in [(1, 200, 1088), (3, 64, 2048), (8, 257, 3072), (11, 136, 576), (16, 520, 1024)]:
        case = make(m, n, k, bits, dtype, epi, seed=m * 7 + bits)
        assert_close(run_case(case, m, n, k, bits, dtype, epi), case["out"], dtype)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("nk", [(5120, 5120), (1024, 5120), (25600, 5120), (5120, 25600), (151936, 5120)])
def test_config2_shapes_sampled(bits, nk):
    """Full config-2 shapes on the GPU (the 151936 x 5120 LM head included: its own two-CTA-per-SM
    plan); the oracle checks a random sample of output rows."""
    S = smallm()
    n, k = nk
    rng = np.random.default_rng(n + k + bits)
    sample = np.sort(rng.choice(n, size=min(n, 384), replace=False))
    # codes drawn directly (the GEMM does not care how they were produced), scales/biases of
    # the size a N(0, 0.02) weight gives
    packed = rng.integers(0, 2 ** 32, size=(n, k * bits // 32), dtype=np.uint32)
    span = 0.1 / ((1 << bits) - 1)
    sc = A.to_storage((span * (0.5 + rng.random((n, k // 64)))).astype(np.float32), "bf16")
    bi = A.to_storage((-0.05 * (0.5 + rng.random((n, k // 64)))).astype(np.float32), "bf16")
    for m in (1, 2, 4, 5, 8, 9, 16):
        x = A.to_storage(rng.standard_normal((m, k)).astype(np.float32), "bf16")
        out = S.matmul(dev(x), S.Weights(dev(packed), dev(sc), dev(bi), bits))
        torch.cuda.synchronize()
        got = host(out)[:, sample]
        ref = A.qgemm(x, packed[sample], sc[sample], bi[sample], bits=bits)
        assert_close(got, ref, "bf16")


@pytest.mark.parametrize("bits", [0, 4, 8])
@pytest.mark.parametrize("n,k", [(5120, 5120), (7168, 5120), (2048, 6144), (96, 512), (25600, 5120)])
def test_batch_invariance_bitwise(bits, n, k):
    """Each row of an M-row call equals the same row computed alone (verify == greedy); the
    int4 (25600, 5120) case runs two CTAs per SM, its M > 8 form in two waves."""
    S = smallm()
    torch.manual_seed(1)
    if bits:
        p, sc, bi = A.quantize((np.random.default_rng(2).standard_normal((n, k)) * 0.02).astype(np.float32), bits)
        w = S.Weights(dev(p), dev(sc), dev(bi), bits)
    else:
        w = S.Weights((torch.randn(n, k, device="cuda") * 0.02).to(torch.bfloat16))
    x = torch.randn(16, k, device="cuda").to(torch.bfloat16)
    res = torch.randn(16, n, device="cuda").to(torch.bfloat16)
    singles = [S.matmul(x[i:i + 1], w, epilogue="residual", residual=res[i:i + 1]) for i in range(16)]
    for m in (2, 5, 9, 16):
        batch = S.matmul(x[:m], w, epilogue="residual", residual=res[:m])
        for i in range(m):
            assert torch.equal(batch[i].view(torch.int16), singles[i][0].view(torch.int16)), (m, i)


def test_writes_stay_inside_output_and_workspace_is_reusable():
    S = smallm()
    n, k, m = 1000, 2048, 7
    p, sc, bi = A.quantize((np.random.default_rng(3).standard_normal((n, k)) * 0.02).astype(np.float32), 4)
    w = S.Weights(dev(p), dev(sc), dev(bi), 4)
    x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    canary = torch.full((m * n + 4096,), 12345.0, device="cuda").to(torch.bfloat16)
    out = canary[:m * n].view(m, n)
    ws_bytes = S.workspace_size(m, n, k, torch.bfloat16, 4)
    ws = torch.zeros(max(ws_bytes, 256) // 4 + 64, dtype=torch.int32, device="cuda")
    r1 = S.matmul(x, w, out=out, workspace=ws).clone()
    r2 = S.matmul(x, w, out=out, workspace=ws).clone()
    torch.cuda.synchronize()
    assert torch.equal(r1.view(torch.int16), r2.view(torch.int16))
    assert torch.all(canary[m * n:] == 12345.0)
    ref = A.qgemm(host(x), p, sc, bi, bits=4)
    assert_close(host(r1), ref, "bf16")


def test_workspace_shared_across_shapes():
    """A GEMM with many split-K row blocks (counters past the first 256 bytes) alternating on
    one workspace with a GEMM of few row blocks (partials early in the workspace): neither
    corrupts the other's ticket counters."""
    S = smallm()
    rng = np.random.default_rng(21)
    shapes = [(20000, 2048), (256, 4096), (7168, 5120)]
    mats = []
    for n, k in shapes:
        p = rng.integers(0, 2 ** 32, size=(n, k // 8), dtype=np.uint32)
        sc = A.to_storage((0.005 * (0.5 + rng.random((n, k // 64)))).astype(np.float32), "bf16")
        bi = A.to_storage((-0.04 * (0.5 + rng.random((n, k // 64)))).astype(np.float32), "bf16")
        x = A.to_storage(rng.standard_normal((5, k)).astype(np.float32), "bf16")
        mats.append((p, sc, bi, x, S.Weights(dev(p), dev(sc), dev(bi), 4), dev(x)))
    need = max(S.workspace_size(5, n, k, torch.bfloat16, 4) for n, k in shapes)
    assert all(S.workspace_size(5, n, k, torch.bfloat16, 4) > 0 for n, k in shapes)
    ws = torch.zeros(need // 4 + 64, dtype=torch.int32, device="cuda")
    refs = [A.qgemm(x, p, sc, bi, bits=4) for p, sc, bi, x, _, _ in mats]
    for rnd in range(3):
        for (p, sc, bi, x, w, xd), ref in zip(mats, refs):
            out = S.matmul(xd, w, workspace=ws)
            torch.cuda.synchronize()
            assert_close(host(out), ref, "bf16")


def test_empty_batch_and_unsupported():
    S = smallm()
    p, sc, bi = A.quantize(np.zeros((64, 512), np.float32), 4)
    w = S.Weights(dev(p), dev(sc), dev(bi), 4)
    out = S.matmul(torch.zeros(0, 512, device="cuda", dtype=torch.bfloat16), w)
    assert out is not None and out.shape == (0, 64)
    # K mismatch -> None (the caller keeps its own path), like SmallMGEMM.matmul's nil
    assert S.matmul(torch.zeros(2, 448, device="cuda", dtype=torch.bfloat16), w) is None
    # dtype mismatch between x and scales -> None
    assert S.matmul(torch.zeros(2, 512, device="cuda", dtype=torch.float16), w) is None


def test_large_m_tensor_core_rows_invariant():
    """M > 16 runs on the tensor cores; a row depends only on its own activations."""
    S = smallm()
    n, k = 320, 1024
    p, sc, bi = A.quantize((np.random.default_rng(4).standard_normal((n, k)) * 0.02).astype(np.float32), 8)
    w = S.Weights(dev(p), dev(sc), dev(bi), 8)
    x = A.to_storage(np.random.default_rng(5).standard_normal((300, k)).astype(np.float32), "bf16")
    out = S.matmul(dev(x), w)
    torch.cuda.synchronize()
    assert_close(host(out), A.qgemm(x, p, sc, bi, bits=8), "bf16")
    # row 137 of 300 (second token tile) == row 17 of 40 (first tile) == row 117 of 200
    other = S.matmul(dev(x)[120:160], w)
    third = S.matmul(dev(x)[20:220], w)
    assert torch.equal(out[137].view(torch.int16), other[17].view(torch.int16))
    assert torch.equal(out[137].view(torch.int16), third[117].view(torch.int16))


@pytest.mark.parametrize("bits", [0, 4, 8])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("epi", ["none", "bias", "residual", "biasResidual", "siluGate", "biasGelu",
                                 "biasGeluResidual"])
def test_tensor_core_every_class(bits, dtype, epi):
    """Calls above 16 rows (tcgen05 path): partial token tiles, N not a multiple of 128,
    fewer K stages than pipeline stages, and several token tiles."""
    for m, n, k in [(17, 200, 1088), (40, 64, 128), (130, 257, 576), (300, 136, 2048)]:
        case = make(m, n, k, bits, dtype, epi, seed=m * 5 + bits)
        assert_close(run_case(case, m, n, k, bits, dtype, epi), case["out"], dtype)


@pytest.mark.parametrize("bits", [0, 4, 8])
@pytest.mark.parametrize("epi", ["none", "biasResidual", "siluGate", "biasGeluResidual"])
def test_tensor_core_k_splits(bits, epi):
    """Calls of at most 256 rows with few row tiles split K over CTAs (N 256, K 4096: 4 splits;
    N 200, K 2560: 2 uneven splits; N 136, K 3072: 3): each split's fp32 sums go through the
    workspace and the tile's last split adds them in split order, then runs the epilogue.
    Against the oracle, one and two token tiles, and above 256 rows (one split)."""
    for m, n, k in [(40, 256, 4096), (130, 200, 2560), (250, 136, 3072), (300, 136, 3072)]:
        case = make(m, n, k, bits, "bf16", epi, seed=m * 3 + bits)
        assert_close(run_case(case, m, n, k, bits, "bf16", epi), case["out"], "bf16")


def test_tensor_core_k_split_rows_invariant():
    """The split count depends on (N, K) and the row class only: a row's value is the same at
    every M of 17-256 rows, and at every M above 256."""
    S = smallm()
    n, k = 256, 4096
    p, sc, bi = A.quantize((np.random.default_rng(6).standard_normal((n, k)) * 0.02).astype(np.float32), 4)
    w = S.Weights(dev(p), dev(sc), dev(bi), 4)
    x = A.to_storage(np.random.default_rng(7).standard_normal((300, k)).astype(np.float32), "bf16")
    out = S.matmul(dev(x), w)
    other = S.matmul(dev(x)[120:160], w)
    third = S.matmul(dev(x)[20:220], w)
    big = S.matmul(dev(x)[0:280], w)
    torch.cuda.synchronize()
    assert_close(host(out), A.qgemm(x, p, sc, bi, bits=4), "bf16")
    assert_close(host(third), A.qgemm(x[20:220], p, sc, bi, bits=4), "bf16")
    assert torch.equal(third[117].view(torch.int16), other[17].view(torch.int16))
    assert torch.equal(out[137].view(torch.int16), big[137].view(torch.int16))


def test_tensor_core_config2_shape_sampled():
    """A prefill-sized call (M 256, N 25600, K 5120, int4) against sampled oracle rows."""
    S = smallm()
    n, k, m = 25600, 5120, 256
    rng = np.random.default_rng(77)
    sample = np.sort(rng.choice(n, size=256, replace=False))
    packed = rng.integers(0, 2 ** 32, size=(n, k // 8), dtype=np.uint32)
    span = 0.1 / 15
    sc = A.to_storage((span * (0.5 + rng.random((n, k // 64)))).astype(np.float32), "bf16")
    bi = A.to_storage((-0.05 * (0.5 + rng.random((n, k // 64)))).astype(np.float32), "bf16")
    x = A.to_storage(rng.standard_normal((m, k)).astype(np.float32), "bf16")
    out = S.matmul(dev(x), S.Weights(dev(packed), dev(sc), dev(bi), 4))
    torch.cuda.synchronize()
    got = host(out)[:, sample]
    ref = A.qgemm(x, packed[sample], sc[sample], bi[sample], bits=4)
    assert_close(got, ref, "bf16")
