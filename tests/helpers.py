"""Shared helpers for the parity tests."""
from __future__ import annotations

import numpy as np
import torch


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    """BF16 tensor -> numpy uint16 bit patterns (on CPU)."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def bits_to_bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(torch.bfloat16)


def np_(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().numpy()


def bf16_ulp_distance(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """Distance in BF16 ulps between two bit-pattern arrays (ordered integer map)."""
    def ordered(bits):
        v = bits.astype(np.int32)
        return np.where(v & 0x8000, 0x8000 - (v & 0x7FFF), 0x8000 + (v & 0x7FFF))
    return np.abs(ordered(a_bits) - ordered(b_bits))


def assert_codes_close(q_gpu: np.ndarray, q_ref: np.ndarray, max_rate: float, what: str) -> float:
    """INT8 codes that may differ by at most 1 at a documented rate (CPU oracle:
    IEEE division instead of the GPU's fast division)."""
    diff = np.abs(q_gpu.astype(np.int32) - q_ref.astype(np.int32))
    assert diff.max(initial=0) <= 1, f"{what}: code differs by {diff.max()}"
    rate = float((diff != 0).mean()) if diff.size else 0.0
    assert rate <= max_rate, f"{what}: code mismatch rate {rate:.2e} > {max_rate:.1e}"
    return rate
