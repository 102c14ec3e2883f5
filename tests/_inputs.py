"""Seeded synthetic inputs for the attention path (numpy, Philox4x32-10).

Every tensor is drawn from its own counter-based stream keyed by
(seed, tensor id), so any tensor can be regenerated independently.  fp16
values are rounded to nearest even (numpy's float16 conversion).  The
distributions follow the benchmark configs: Q/K/V ~ N(0,1); DeltaNet q and k
L2-normalised per head (q also scaled by 1/sqrt(dk), as
lib/Models/Qwen35/Qwen35ModelBuilder.cpp:155-157 does), beta =
half(sigmoid(N(0,1))), decay = exp(-softplus(N(0,1))), states ~ N(0, 0.02).
"""
from __future__ import annotations

import numpy as np

DEFAULT_SEED = 179531  # the seed of the reference's FlashAttentionTest


def stream(seed: int, tensor_id: int) -> np.random.Generator:
    return np.random.Generator(np.random.Philox(key=[seed & (2**64 - 1), tensor_id]))


def normal(seed: int, tensor_id: int, shape, scale: float = 1.0) -> np.ndarray:
    return (stream(seed, tensor_id).standard_normal(shape, dtype=np.float32) * np.float32(scale))


def half_normal(seed: int, tensor_id: int, shape) -> np.ndarray:
    return normal(seed, tensor_id, shape).astype(np.float16)


def gqa_case(batch, tokens, past, query_heads, kv_heads, head_dim, capacity=None, seed=DEFAULT_SEED):
    """Returns q [B,T,Hq,D], k_cache/v_cache [B,cap,Hkv,D] (rows [0,past+T) filled), fp16."""
    capacity = past + tokens if capacity is None else capacity
    q = half_normal(seed, 1, (batch, tokens, query_heads, head_dim))
    k = np.zeros((batch, capacity, kv_heads, head_dim), np.float16)
    v = np.zeros_like(k)
    k[:, :past + tokens] = half_normal(seed, 2, (batch, past + tokens, kv_heads, head_dim))
    v[:, :past + tokens] = half_normal(seed, 3, (batch, past + tokens, kv_heads, head_dim))
    return q, k, v


def _l2(x: np.ndarray, scale: float) -> np.ndarray:
    x = x.astype(np.float32)
    s = np.sum(x * x, axis=-1, keepdims=True, dtype=np.float32)
    return (x * (np.float32(scale) / np.sqrt(s + np.float32(1e-6)))).astype(np.float32)


def softplus(x: np.ndarray) -> np.ndarray:
    return np.logaddexp(np.float32(0), x).astype(np.float32)


def delta_case(batch, tokens, key_heads, key_dim, value_heads, value_dim, state_std=0.0,
               seed=DEFAULT_SEED):
    """Returns dict(q, k [B,T,Hk*dk] f32; v [B,T,Hv*dv] f16; beta, decay [B,T,Hv] f32;
    state [B,Hv,dk,dv] f32)."""
    qr = normal(seed, 11, (batch, tokens, key_heads, key_dim))
    kr = normal(seed, 12, (batch, tokens, key_heads, key_dim))
    q = _l2(qr, 1.0 / np.sqrt(key_dim)).reshape(batch, tokens, key_heads * key_dim)
    k = _l2(kr, 1.0).reshape(batch, tokens, key_heads * key_dim)
    v = half_normal(seed, 13, (batch, tokens, value_heads * value_dim))
    beta = (1.0 / (1.0 + np.exp(-normal(seed, 14, (batch, tokens, value_heads))))).astype(np.float16).astype(np.float32)
    decay = np.exp(-softplus(normal(seed, 15, (batch, tokens, value_heads)))).astype(np.float32)
    if state_std:
        state = normal(seed, 16, (batch, value_heads, key_dim, value_dim), state_std)
    else:
        state = np.zeros((batch, value_heads, key_dim, value_dim), np.float32)
    return dict(q=q, k=k, v=v, beta=beta, decay=decay, state=state)


def errors(actual, expected) -> tuple[float, float]:
    """(max-abs error, relative L2 error) in float64."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    diff = a - e
    denom = np.linalg.norm(e.ravel())
    return float(np.max(np.abs(diff))), float(np.linalg.norm(diff.ravel()) / max(denom, 1e-300))


# The acceptance bar: max-abs <= 1e-2 and
# relative L2 <= 2e-3 on attention outputs and on the updated DeltaNet state.
MAX_ABS = 1e-2
REL_L2 = 2e-3
