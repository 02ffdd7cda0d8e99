"""vella_qgemm_noalloc, the GEMM entry point that allocates nothing.

Callers that cannot allocate device memory (code running during CUDA graph capture, a
real-time audio thread that must not block on an allocation, an embedder whose device
memory belongs to another allocator) use this entry point: its split-K scratch is a static
device array inside the library.  This test calls it through the C ABI twice in a row and
checks each result against vella_qgemm's on the same inputs.  The file sorts last so a
run that stops at the first failure has run every other test before it; it also passes
on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import affine as A
from tests._util import dev, host

pytestmark = pytest.mark.gpu

REL = 1e-2


def _lib():
    from vella_b200 import _lib as L
    L.declare("vella_qgemm_noalloc", ctypes.c_int,
              [ctypes.POINTER(L.QgemmDesc)] + [ctypes.c_void_p] * 10 + [ctypes.c_void_p])
    return L


@pytest.mark.parametrize("bits,m,n,k,epi", [
    (4, 5, 5120, 5120, "residual"),   # split-K: uses the static scratch
    (8, 9, 2048, 6144, "none"),
    (4, 3, 1000, 2048, "siluGate"),
])
def test_noalloc_matches_qgemm_on_two_calls(bits, m, n, k, epi):
    L = _lib()
    lib = L.lib()
    rng = np.random.default_rng(11)
    p, sc, bi = A.quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32), bits)
    up = A.quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32), bits) if epi == "siluGate" else None
    w, s, b = dev(p), dev(sc), dev(bi)
    uw, us, ub = (dev(up[0]), dev(up[1]), dev(up[2])) if up else (None, None, None)
    res = torch.randn(m, n, device="cuda").to(torch.bfloat16) if epi == "residual" else None
    d = L.QgemmDesc(m, n, k, bits, 64, L.BF16, L.EPI[epi])
    assert L.lib().vella_qgemm_workspace_size(ctypes.byref(d)) > 0 or epi != "residual"
    stream = torch.cuda.current_stream().cuda_stream
    ws_bytes = lib.vella_qgemm_workspace_size(ctypes.byref(d))
    ws = torch.zeros(max(ws_bytes, 256) // 4 + 64, dtype=torch.int32, device="cuda")
    for call in range(2):
        x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
        ref = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        got = torch.full((m, n), float("nan"), device="cuda", dtype=torch.bfloat16)
        ptrs = [x.data_ptr(), w.data_ptr(), s.data_ptr(), b.data_ptr(), L.ptr(uw), L.ptr(us), L.ptr(ub),
                None, L.ptr(res)]
        L.check(lib.vella_qgemm(ctypes.byref(d), *ptrs, ref.data_ptr(), ws.data_ptr(), ws_bytes, stream))
        L.check(lib.vella_qgemm_noalloc(ctypes.byref(d), *ptrs, got.data_ptr(), stream))
        torch.cuda.synchronize()
        g, r = host(got), host(ref)
        gf, rf = A.from_storage(g, "bf16"), A.from_storage(r, "bf16")
        assert np.isfinite(gf).all(), call
        assert A.relative_rms(gf, rf) <= REL, call
        assert np.abs(gf - rf).max() <= REL * max(np.abs(rf).max(), 1e-6), call
        # same kernel, same plan, same split order: the results agree bit for bit
        assert np.array_equal(g, r), call


def test_noalloc_rejects_shapes_beyond_its_scratch():
    L = _lib()
    # an lm_head-sized GEMM at 16 rows with K = 25664 (not a multiple of 512: the split-K
    # register kernel) needs far more than the 32 MiB static array
    d = L.QgemmDesc(16, 151936, 25664, 4, 64, L.BF16, 0)
    assert L.lib().vella_qgemm_workspace_size(ctypes.byref(d)) > 32 << 20
    x = torch.zeros(8, device="cuda")
    rc = L.lib().vella_qgemm_noalloc(ctypes.byref(d), *([x.data_ptr()] * 4), None, None, None, None, None,
                                     x.data_ptr(), None)
    assert rc == L.E_INVALID
    assert "static array" in L.last_error()
