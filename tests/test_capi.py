"""The C-ABI library loads here (no GPU needed) and exports every function the public
headers declare; pure queries answer without touching a device."""
import ctypes
import glob
import os
import re
import subprocess

import pytest

from vella_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"^[A-Za-z_][\w \*]*?\b(vella_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_functions()
    assert "vella_qgemm" in names and "vella_last_error" in names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (vella_\w+)", out))
    assert set(names) <= exported
    # nothing else with C linkage leaks out of the library
    assert exported == set(names), sorted(exported - set(names))


def test_version_and_last_error():
    lib = _lib.lib()
    assert lib.vella_version().decode().startswith("vella-b200")
    assert isinstance(_lib.last_error(), str)


@pytest.mark.parametrize("m,n,k,bits,epi,ok", [
    (1, 5120, 5120, 4, "none", True),
    (16, 151936, 5120, 4, "none", True),
    (9, 25600, 5120, 8, "siluGate", True),
    (4, 96, 512, 0, "bias", True),
    (256, 64, 448, 4, "residual", True),
    (257, 64, 448, 4, "none", True),    # above 16 rows: the tensor-core kernel
    (1500, 1280, 1280, 0, "bias", True),
    (4, 96, 520, 4, "none", False),     # K not a multiple of the group
    (4, 96, 512, 5, "none", False),     # unsupported bit width
    (0, 96, 512, 4, "none", True),      # empty batch is a no-op
])
def test_supports_is_a_pure_query(m, n, k, bits, epi, ok):
    d = _lib.QgemmDesc(m, n, k, bits, 64, _lib.BF16, _lib.EPI[epi])
    assert bool(_lib.lib().vella_qgemm_supports(ctypes.byref(d))) == ok


def test_group_size_and_dtype_checked():
    L = _lib.lib()
    assert not L.vella_qgemm_supports(ctypes.byref(_lib.QgemmDesc(1, 64, 512, 4, 32, _lib.BF16, 0)))
    assert not L.vella_qgemm_supports(ctypes.byref(_lib.QgemmDesc(1, 64, 512, 4, 64, 7, 0)))
    assert L.vella_qgemm_supports(ctypes.byref(_lib.QgemmDesc(1, 64, 512, 4, 64, _lib.F16, 0)))


def test_workspace_depends_on_shape_not_rows():
    L = _lib.lib()
    # the split plan is a function of (N, K, bits, gate); workspace grows with ceil(M/16) only
    sizes = [L.vella_qgemm_workspace_size(ctypes.byref(_lib.QgemmDesc(m, 5120, 5120, 4, 64, _lib.BF16, 0)))
             for m in (1, 8, 16)]
    assert sizes[0] == sizes[1] == sizes[2] > 0


def test_tensor_core_k_split_workspace_follows_the_row_classes():
    """Calls of 17-256 rows whose row tiles leave SMs idle split K and need fp32 partial sums in
    the workspace; calls of more than 256 rows, and shapes whose row tiles fill the GPU, do not.
    The split count (hence each row's value) depends on N and K only within a class."""
    L = _lib.lib()

    def ws(m, n, k, bits=4, epi=0):
        return L.vella_qgemm_workspace_size(ctypes.byref(_lib.QgemmDesc(m, n, k, bits, 64, _lib.BF16, epi)))

    # bf16 draft down projection (16 row tiles, 96 stages): four splits below 257 rows
    assert ws(32, 2048, 6144, 0) > 0 and ws(256, 2048, 6144, 0) > 0
    assert ws(257, 2048, 6144, 0) == 0 and ws(1088, 2048, 6144, 0) == 0
    # int4 down projection of the 30B target (K = 25600): three splits for the long K
    assert ws(160, 5120, 25600) > 0 and ws(300, 5120, 25600) == 0
    # the target's gate/up and LM head: their row tiles fill the GPU, one split
    assert ws(160, 25600, 5120, 4, _lib.EPI["siluGate"]) == 0
    assert ws(160, 151936, 5120) == 0
    # the fp32 sums are sized for the rows rounded up to one 256-token tile
    assert ws(32, 2048, 6144, 0) == ws(256, 2048, 6144, 0) >= 4 * 256 * 2048 * 4


def test_unsupported_call_returns_status_not_crash():
    L = _lib.lib()
    d = _lib.QgemmDesc(4, 96, 520, 4, 64, _lib.BF16, 0)
    rc = L.vella_qgemm(ctypes.byref(d), *([None] * 10), None, 0, None)
    assert rc == _lib.E_UNSUPPORTED
    assert "unsupported" in _lib.last_error()
    d = _lib.QgemmDesc(4, 96, 512, 4, 64, _lib.BF16, 0)
    rc = L.vella_qgemm(ctypes.byref(d), *([None] * 10), None, 0, None)
    assert rc == _lib.E_INVALID
