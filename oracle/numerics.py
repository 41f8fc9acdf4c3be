"""Rounding helpers and the elementary functions the reference trunk uses (oracle only)."""

from __future__ import annotations

import numpy as np
from scipy.special import erf


def round_bf16(values: np.ndarray) -> np.ndarray:
    """Round to the nearest bfloat16 (ties to even), returned as float32.

    The input is first rounded to float32, which is what a float32 accumulator
    holds before the kernels narrow it.
    """

    f32 = np.ascontiguousarray(np.asarray(values, dtype=np.float32))
    bits = f32.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    return rounded.astype(np.uint32).view(np.float32).reshape(f32.shape)


def round_to(values: np.ndarray, storage: str) -> np.ndarray:
    """Round to a storage dtype ("fp32", "fp16", "bf16") and return float64."""

    if storage == "fp32":
        return np.asarray(values, dtype=np.float32).astype(np.float64)
    if storage == "fp16":
        return np.asarray(values, dtype=np.float32).astype(np.float16).astype(np.float64)
    if storage == "bf16":
        return round_bf16(values).astype(np.float64)
    raise ValueError(f"Unknown storage {storage!r}.")


def layer_norm(x: np.ndarray, weight: np.ndarray, bias: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """torch.nn.LayerNorm over the last axis (biased variance), as trunk.py:133,138,270 use it."""

    mean = x.mean(axis=-1, keepdims=True)
    centered = x - mean
    var = (centered * centered).mean(axis=-1, keepdims=True)
    return centered / np.sqrt(var + eps) * weight + bias


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """RMSNorm with a gain only (cardgym/nn/trunk.py:104-115): x * rsqrt(mean(x^2) + eps) * g."""

    return x / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps) * weight


def gelu(x: np.ndarray) -> np.ndarray:
    """Exact (erf) GELU, nn.GELU()'s default (cardgym/nn/trunk.py:139, cardgym/nn/model.py:12-17)."""

    return 0.5 * x * (1.0 + erf(x / np.sqrt(2.0)))
