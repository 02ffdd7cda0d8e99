"""Host mirror of the reference's kernel-library seam ``SmallMGEMM`` over the CUDA library.

Reference: ``Worker/Sources/SmallMGEMM/SmallMGEMM.swift``
  * ``matmul(x, weights, epilogue:)`` (:126-207) returns ``nil`` when the call is not
    handled; ``matmul`` here returns ``None`` in the same cases, and the caller keeps its
    own path (``y = matmul(x, w) or stock(x)``).
  * ``supports(m:n:k:dtype:format:epilogue:)`` (:113-120) is a pure query.
  * ``Weights`` / ``WeightFormat`` / ``Epilogue`` (:31-74) become ``Weights`` and the
    ``epilogue``/``bias``/``residual``/``up`` arguments.
  * ``fits`` (:210-227): the weights' arrays must match their format, K and the
    activation dtype, else ``None``.

Tensors are torch CUDA tensors (torch provides device memory and streams only); the work
runs in ``libvella_cuda.so`` on the current torch stream.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib

_DTYPES = {torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}


@dataclass
class Weights:
    """W [N, K]: dense (``bits`` = 0, ``w`` in the activation dtype) or MLX affine
    (``bits`` 4 | 8, ``w`` packed uint32 [N, K*bits/32] viewed as int32, ``scales`` and
    ``biases`` [N, K/64])."""

    w: torch.Tensor
    scales: Optional[torch.Tensor] = None
    biases: Optional[torch.Tensor] = None
    bits: int = 0
    group_size: int = 64

    @property
    def n(self) -> int:
        return self.w.shape[0]

    def k(self) -> int:
        return self.w.shape[1] * (32 // self.bits if self.bits else 1)


def _desc(m, n, k, dtype, bits, epilogue, group=64) -> _lib.QgemmDesc:
    return _lib.QgemmDesc(m, n, k, bits, group, _DTYPES.get(dtype, -1), _lib.EPI[epilogue])


def supports(m: int, n: int, k: int, dtype: torch.dtype, bits: int = 0, epilogue: str = "none") -> bool:
    d = _desc(m, n, k, dtype, bits, epilogue)
    return bool(_lib.lib().vella_qgemm_supports(ctypes.byref(d)))


def _fits(w: Weights, k: int, dtype: torch.dtype) -> bool:
    if w.w.dim() != 2 or not w.w.is_contiguous():
        return False
    if w.bits == 0:
        return w.w.dtype == dtype and w.w.shape[1] == k
    if w.bits not in (4, 8) or w.group_size != 64 or w.w.dtype not in (torch.int32, torch.uint32):
        return False
    if w.w.shape[1] * 32 // w.bits != k or w.scales is None or w.biases is None:
        return False
    groups = (w.w.shape[0], k // w.group_size)
    return (tuple(w.scales.shape) == groups and tuple(w.biases.shape) == groups
            and w.scales.dtype == dtype and w.biases.dtype == dtype
            and w.scales.is_contiguous() and w.biases.is_contiguous())


def matmul(x: torch.Tensor, weights: Weights, epilogue: str = "none", bias: Optional[torch.Tensor] = None,
           residual: Optional[torch.Tensor] = None, up: Optional[Weights] = None,
           out: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
    """out[..., N] = epilogue(x[..., K] . W^T), or None when the call is not handled."""
    k = x.shape[-1]
    n = weights.n
    rows = x.numel() // max(k, 1)
    if not x.is_cuda or x.dtype not in _DTYPES or not _fits(weights, k, x.dtype):
        return None
    if epilogue in ("bias", "biasResidual", "biasGelu", "biasGeluResidual") and (bias is None or bias.numel() != n):
        return None
    if epilogue in ("residual", "biasResidual", "biasGeluResidual") and (residual is None or residual.numel() != rows * n):
        return None
    if epilogue == "siluGate":
        if up is None or up.bits != weights.bits or up.w.shape != weights.w.shape or not _fits(up, k, x.dtype):
            return None
    d = _desc(rows, n, k, x.dtype, weights.bits, epilogue, weights.group_size)
    L = _lib.lib()
    if not L.vella_qgemm_supports(ctypes.byref(d)):
        return None
    x2 = x.reshape(rows, k).contiguous()
    if out is None:
        out = torch.empty(*x.shape[:-1], n, dtype=x.dtype, device=x.device)
    res = residual.reshape(rows, n).contiguous() if residual is not None else None
    u = up if up is not None else Weights(None)
    ws_ptr, ws_bytes = (workspace.data_ptr(), workspace.numel() * workspace.element_size()) if workspace is not None else (None, 0)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    _lib.check(L.vella_qgemm(ctypes.byref(d), x2.data_ptr(), weights.w.data_ptr(), _lib.ptr(weights.scales),
                             _lib.ptr(weights.biases), _lib.ptr(u.w), _lib.ptr(u.scales), _lib.ptr(u.biases),
                             _lib.ptr(bias), _lib.ptr(res), out.data_ptr(), ws_ptr, ws_bytes, stream))
    return out


def workspace_size(m: int, n: int, k: int, dtype: torch.dtype, bits: int = 0, epilogue: str = "none") -> int:
    d = _desc(m, n, k, dtype, bits, epilogue)
    return int(_lib.lib().vella_qgemm_workspace_size(ctypes.byref(d)))
