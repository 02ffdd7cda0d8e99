"""numpy storage arrays (oracle side) <-> torch CUDA tensors (library side)."""
import numpy as np
import torch

TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def dev(a: np.ndarray, dtype: str = None, device="cuda") -> torch.Tensor:
    """Storage array -> device tensor.  bf16 storage is uint16 bit patterns."""
    if a.dtype == np.uint16 and dtype in (None, "bf16"):
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(device)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32).copy()).to(device)
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def host(t: torch.Tensor) -> np.ndarray:
    """Device tensor -> storage array (bf16 as uint16 bits)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.int32:
        return t.numpy().view(np.uint32)
    return t.numpy()


def as_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    from oracle.affine import from_storage
    return from_storage(a, dtype)
