"""Shared helpers for the parity tests (comparison metric of the oracle)."""
import numpy as np


def rel_err(got, ref, floor_frac=1e-3):
    """max |g - r| / max(|r|, floor_frac * max|r|), the parity metric."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    floor = floor_frac * max(float(np.abs(ref).max()), 1e-30)
    return float((np.abs(got - ref) / np.maximum(np.abs(ref), floor)).max())


def norm_err(got, ref):
    """Normwise relative error max|g - r| / max|r| (attention parity metric:
    rounding P to bf16 makes the error absolute relative to the row scale)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(float(np.abs(ref).max()), 1e-30))


def to_np_bf16(t):
    """torch bf16 tensor -> numpy uint16 bit patterns."""
    import torch

    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def from_np_bf16(a, device="cuda"):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(device).view(torch.bfloat16)
