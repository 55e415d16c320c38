"""Helpers shared by the GPU parity tests."""

from __future__ import annotations

import numpy as np
import torch

# North-star tolerances for BF16 layer outputs against the reference path.
MAX_ABS = 2e-2
MIN_COSINE = 0.9999


def bits(t: torch.Tensor) -> np.ndarray:
    """BF16 tensor -> numpy uint16 bit patterns (host copy)."""
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def from_bits(a: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(torch.bfloat16).to(device)


def f32(a_bits: np.ndarray) -> np.ndarray:
    return (np.asarray(a_bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / (na * nb))


def bf16_ulp(v: np.ndarray) -> np.ndarray:
    """Spacing of BF16 values at |v| (2^(e-7) for |v| in [2^e, 2^(e+1)))."""
    a = np.abs(np.asarray(v, dtype=np.float32))
    e = np.floor(np.log2(np.maximum(a, np.float32(2.0 ** -126))))
    return np.exp2(e - 7).astype(np.float32)


def assert_layer_close(gpu_bits: np.ndarray, ref_bits: np.ndarray, *, max_abs: float = MAX_ABS,
                       min_cos: float = MIN_COSINE, ulps: int = 1) -> dict:
    """BF16 layer tolerance: every element within max(max_abs, one BF16 ulp of
    the reference value) -- above |y| = 4 one ulp is 0.03125, so a single
    rounding flip of a non-bit-identical FP32 sum exceeds 2e-2 -- and
    cosine >= min_cos over the tensor."""
    g, r = f32(gpu_bits), f32(ref_bits)
    assert np.isfinite(g).all(), "non-finite GPU output"
    diff = np.abs(g - r)
    err = float(diff.max()) if g.size else 0.0
    bound = np.maximum(np.float32(max_abs), np.float32(ulps) * bf16_ulp(r))
    worst = float((diff / bound).max()) if g.size else 0.0
    cos = cosine(g, r)
    same = float((np.asarray(gpu_bits) == np.asarray(ref_bits)).mean()) if g.size else 1.0
    over = int((diff > max_abs).sum())
    assert worst <= 1.0, f"max-abs {err} exceeds max({max_abs}, {ulps} BF16 ulp) (worst ratio {worst:.3f})"
    assert cos >= min_cos, f"cosine {cos} < {min_cos}"
    return {"max_abs": err, "cosine": cos, "bit_identical": same, "over_max_abs_within_ulp": over}


def bank_host(bank, ids=None):
    """Host copies of the bank tensors (optionally only the experts in ids,
    re-indexed 0..len(ids)-1)."""
    ts = (bank.gate_up_weight, bank.gate_up_scale_inv, bank.down_weight, bank.down_scale_inv)
    if ids is not None:
        sel = torch.as_tensor(np.asarray(ids, dtype=np.int64), device=bank.gate_up_weight.device)
        ts = tuple(t.index_select(0, sel) for t in ts)
    return tuple(t.cpu().numpy() for t in ts)


def shared_host(shared_tensors):
    return None if shared_tensors is None else tuple(t.cpu().numpy() for t in shared_tensors)
