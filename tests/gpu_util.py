"""Helpers shared by the GPU parity tests."""
import numpy as np
import torch

TORCH = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def dev(a, dtype=None):
    """numpy -> contiguous CUDA tensor (uint32 kept as torch.uint32)."""
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda().contiguous()


def host(t):
    """CUDA tensor -> numpy (16-bit floats widened to float32)."""
    t = t.detach().cpu()
    if t.dtype in (torch.float16, torch.bfloat16):
        t = t.float()
    return t.numpy()


def round_to(a, dtype):
    """float32 numpy array rounded through a torch dtype (bf16/f16) and back."""
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dtype).float().numpy()


def max_rel_err(got, ref, floor=0.0):
    """max |got - ref| / max(|ref|, floor) over all elements (0 where both are 0)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    diff = np.abs(got - ref)
    den = np.maximum(np.abs(ref), floor)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = np.where(diff == 0, 0.0, diff / den)
    return float(np.nanmax(r)) if r.size else 0.0


def bits_equal(a, b):
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    return a.shape == b.shape and a.dtype == b.dtype and np.array_equal(a.view(np.uint8), b.view(np.uint8))
