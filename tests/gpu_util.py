"""Helpers shared by the GPU tests: numpy <-> torch CUDA tensors (bf16 as raw bits)."""
import numpy as np


def dev(a: np.ndarray, bf16: bool = False):
    import torch
    if bf16:
        assert a.dtype == np.uint16
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).cuda()
    return torch.from_numpy(np.ascontiguousarray(a).copy()).cuda()


def host(t) -> np.ndarray:
    import torch
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).cpu().numpy().view(np.uint16)
    return t.detach().cpu().numpy()


def bf16_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max |got - ref| / max |ref| (normwise relative error)."""
    return float(np.abs(got.astype(np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))
