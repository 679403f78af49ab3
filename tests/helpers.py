"""Conversions and comparison helpers shared by the tests."""

from __future__ import annotations

import numpy as np
import torch


def to_u16(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor (any device) -> uint16 bit patterns as numpy."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def from_u16(a: np.ndarray, device="cpu") -> torch.Tensor:
    """uint16 bit patterns -> bf16 tensor."""
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def bf16_compare(got: np.ndarray, want: np.ndarray, atol=1e-2, rtol=1e-2) -> dict:
    """allclose-style comparison of two bf16 arrays (uint16 bit patterns)."""
    g = bf16_to_f32(got).astype(np.float64)
    w = bf16_to_f32(want).astype(np.float64)
    diff = np.abs(g - w)
    return {
        "allclose": bool(np.all(diff <= atol + rtol * np.abs(w))),
        "max_abs": float(diff.max()) if diff.size else 0.0,
        "bit_mismatch": int((got != want).sum()),
        "n": int(got.size),
    }
