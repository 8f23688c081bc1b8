"""Shared helpers for the parity tests."""
from __future__ import annotations

import numpy as np

import oracle as O

# Tolerance stated by the path's contract for bf16 outputs against the
# reference MLX nvfp4 path (float32-accumulating CPU oracle): max-abs 2e-2 and
# mean relative (sum|a-b| / sum|b|) 1e-3.
MAX_ABS = 2e-2
MEAN_REL = 1e-3


def close_stats(actual: np.ndarray, expected: np.ndarray):
    a = np.asarray(actual, np.float64)
    b = np.asarray(expected, np.float64)
    d = np.abs(a - b)
    denom = max(np.abs(b).sum(), 1e-30)
    return float(d.max(initial=0.0)), float(d.sum() / denom)


def assert_bf16_close(actual_bits: np.ndarray, expected_bits: np.ndarray, max_abs=MAX_ABS, mean_rel=MEAN_REL,
                      what=""):
    a = O.bf16_to_f32(actual_bits)
    b = O.bf16_to_f32(expected_bits)
    assert np.all(np.isfinite(a)), f"{what}: non-finite output"
    ma, mr = close_stats(a, b)
    assert ma <= max_abs and mr <= mean_rel, f"{what}: max-abs {ma:.3g} (<= {max_abs}), mean-rel {mr:.3g} (<= {mean_rel})"
    return ma, mr


def det_source(shape, salt: int) -> np.ndarray:
    """The reference tests' deterministic source ((i*17+salt)%31-15)/16
    (Tests/MLXFastTests/NVFP4QuantizedMMTests.swift:372-379)."""
    n = int(np.prod(shape))
    i = np.arange(n, dtype=np.int64)
    return ((((i * 17 + salt) % 31) - 15) / 16.0).astype(np.float32).reshape(shape)


def normal_weights(rng, shape, std=0.02):
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def bf16_normal(rng, shape):
    return O.f32_to_bf16(rng.standard_normal(shape, dtype=np.float32))


def to_torch_bf16(bits: np.ndarray, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(device).view(torch.bfloat16)


def from_torch_bf16(t) -> np.ndarray:
    import torch

    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def to_torch_u32(a: np.ndarray, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint32).view(np.int32)).to(device)


def to_torch(a: np.ndarray, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(device)
