"""Shared helpers for the tests (bf16 <-> numpy bit patterns, fixtures)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def t_from_bits(a: np.ndarray, device="cpu") -> torch.Tensor:
    """uint16 bf16 bit patterns -> torch.bfloat16 tensor (exact)."""
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)


def bits_of(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def assert_close(name, got, ref, atol, rtol):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    diff = np.abs(got - ref)
    bad = diff > atol + rtol * np.abs(ref)
    if bad.any():
        i = np.unravel_index(np.argmax(diff), diff.shape)
        raise AssertionError(
            f"{name}: {bad.sum()} of {bad.size} outside atol={atol} rtol={rtol}; "
            f"max_abs={diff.max():.3e} at {i} (got {got[i]:.6f} ref {ref[i]:.6f})"
        )
