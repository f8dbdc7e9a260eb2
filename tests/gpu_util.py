"""Helpers for the -m gpu parity tests (device setup, oracle comparisons)."""
import numpy as np
import torch


def dev():
    if not torch.cuda.is_available():
        raise RuntimeError("gpu tests need a CUDA device (sm_100a)")
    return torch.device("cuda:0")


def rel_l2(a, b) -> float:
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    den = b.norm().item()
    return (a - b).norm().item() / (den if den > 0 else 1.0)


def u8(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.uint8).cpu().numpy()


def bf16_ulp_mismatch(a: torch.Tensor, b: torch.Tensor):
    """(fraction of elements that differ, max difference in bf16 ulps)."""
    ai = a.contiguous().view(torch.int16).cpu().numpy().astype(np.int32)
    bi = b.contiguous().view(torch.int16).cpu().numpy().astype(np.int32)
    # map sign-magnitude to ordered ints
    ai = np.where(ai < 0, -32768 - ai, ai)
    bi = np.where(bi < 0, -32768 - bi, bi)
    d = np.abs(ai - bi)
    return float((d > 0).mean()), int(d.max()) if d.size else 0
