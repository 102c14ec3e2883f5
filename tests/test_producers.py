"""The producer oracles (q/k norm + partial RoPE, causal conv + SiLU, L2Norm,
DeltaGates) pinned against an independent implementation of the same layers:
transformers' Qwen3-Next modeling code (Qwen3NextRMSNorm, rotate_half,
torch_causal_conv1d_update, l2norm and the gate formulas of its gated
DeltaNet).  Installed transformers differs from the version the reference's
own tests pin, so these are a cross-check of the restated semantics
(pairing, positions, (1 + w), history shifting, scales) at fp16 resolution,
not a bit-exact pin.

Also the restatements' own edge cases: steps shorter than the conv history,
the history carried across steps, rows written at an output offset (the
fused cacheAppend), strided q rows.
"""
import numpy as np
import pytest
import torch

import _inputs
import _oracle

qn = pytest.importorskip("transformers.models.qwen3_next.modeling_qwen3_next")


def f16(a):
    return np.asarray(a, np.float32).astype(np.float16)


def ulps(a, b):
    """Distance in fp16 units in the last place."""
    a = np.asarray(a, np.float16).astype(np.float32)
    b = np.asarray(b, np.float16).astype(np.float32)
    scale = np.maximum(np.abs(a), np.abs(b))
    ulp = np.where(scale < 2.0 ** -14, 2.0 ** -24,
                   2.0 ** (np.floor(np.log2(np.maximum(scale, 1e-30))) - 10))
    return np.abs(a - b) / ulp


def hf_norm_rope(x16, weight, past, rotary_dim, theta, eps):
    """Qwen3-Next q/k path in fp16: RMSNorm (1 + w), then partial RoPE on the
    first rotary_dim dims with cos/sin cast to fp16."""
    batch, tokens, heads, d = x16.shape
    norm = qn.Qwen3NextRMSNorm(d, eps)
    with torch.no_grad():
        norm.weight.copy_(torch.from_numpy(weight))
        x = norm(torch.from_numpy(x16))  # fp16 out
        inv_freq = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2, dtype=torch.int64).float()
                                    / rotary_dim))
        pos = torch.arange(past, past + tokens, dtype=torch.float32)
        freqs = pos[:, None] * inv_freq[None, :]
        emb = torch.cat((freqs, freqs), dim=-1)
        cos = emb.cos().to(torch.float16)[None, :, None, :]
        sin = emb.sin().to(torch.float16)[None, :, None, :]
        rot = x[..., :rotary_dim]
        rot = rot * cos + qn.rotate_half(rot) * sin
        return torch.cat((rot, x[..., rotary_dim:]), dim=-1).numpy()


@pytest.mark.parametrize("tokens,past,heads,d,rot", [(5, 0, 4, 256, 64), (3, 1000, 2, 128, 128),
                                                     (7, 37, 3, 64, 32), (16, 8000, 2, 256, 64)])
def test_norm_rope_matches_transformers(tokens, past, heads, d, rot):
    x = _inputs.half_normal(7, 1, (1, tokens, heads, d))
    w = _inputs.normal(7, 2, (d,), 0.1)
    got = _oracle.norm_rope(x, w, past, rot, 10_000_000.0)
    ref = hf_norm_rope(x, w, past, rot, 10_000_000.0, 1e-6)
    # Rounding points agree.  The sum order, and the phase taken as a division
    # by a power versus a product with a reciprocal (apart by an fp32 ulp of a
    # phase that grows with the position), move a few cos/sin values by one
    # fp16 ulp: results then differ by about one fp16 ulp at unit scale.
    assert np.isfinite(got.astype(np.float32)).all()
    g32, r32 = got.astype(np.float32), ref.astype(np.float32)
    assert (ulps(got, ref) > 0).mean() <= 0.01
    assert np.all(np.abs(g32 - r32) <= 2.0 ** -9 * np.maximum(1.0, np.abs(r32)))


def test_partial_rope_is_norm_rope_without_norm():
    x = _inputs.half_normal(8, 1, (2, 4, 2, 64))
    got = _oracle.norm_rope(x, None, 12, 32, 10000.0)
    # Dims past the rotary width pass through unchanged.
    np.testing.assert_array_equal(got[..., 32:].view(np.uint16), x[..., 32:].view(np.uint16))
    # Position 0 (cos 1, sin 0) leaves a row unchanged.
    first = _oracle.norm_rope(x[:, :1], None, 0, 32, 10000.0)
    np.testing.assert_array_equal(first.view(np.uint16), x[:, :1].view(np.uint16))


def test_norm_rope_writes_at_output_start_with_strided_rows():
    # q sliced from [q | gate] rows (headStride 2D); keys written into a
    # cache at row `past` (the step's cacheAppend).
    d, heads, tokens, past = 64, 2, 3, 5
    qg = _inputs.half_normal(9, 1, (1, tokens, heads, 2 * d))
    w = _inputs.normal(9, 2, (d,), 0.1)
    cache = _inputs.half_normal(9, 3, (1, past + tokens + 2, heads, d))
    got = _oracle.norm_rope(qg, w, past, 32, 10000.0, head_dim=d, output=cache, output_start=past)
    dense = _oracle.norm_rope(np.ascontiguousarray(qg[..., :d]), w, past, 32, 10000.0)
    np.testing.assert_array_equal(got[:, past:past + tokens].view(np.uint16), dense.view(np.uint16))
    np.testing.assert_array_equal(got[:, :past].view(np.uint16), cache[:, :past].view(np.uint16))
    np.testing.assert_array_equal(got[:, past + tokens:].view(np.uint16),
                                  cache[:, past + tokens:].view(np.uint16))


def hf_conv(x16, w16, hist16):
    """torch_causal_conv1d_update (SiLU) in fp32 on the fp16 values."""
    x = torch.from_numpy(x16.astype(np.float32)).transpose(1, 2).contiguous()  # [B, C, T]
    state = torch.from_numpy(hist16.astype(np.float32)).clone()  # [B, C, K-1]
    w = torch.from_numpy(w16.astype(np.float32))
    out = qn.torch_causal_conv1d_update(x, state, w)
    return out.transpose(1, 2).numpy(), state.numpy()


@pytest.mark.parametrize("tokens", [1, 2, 9])
def test_causal_conv_matches_transformers(tokens):
    batch, channels, k = 2, 48, 4
    x = _inputs.half_normal(10, 1, (batch, tokens, channels))
    w = f16(_inputs.normal(10, 2, (channels, k), 0.5))
    hist = _inputs.half_normal(10, 3, (batch, channels, k - 1))
    got, got_hist = _oracle.causal_conv(x, w, hist, True)
    ref, ref_hist = hf_conv(x, w, hist)
    # Same taps and history; the reference rounds the sum to fp16 before SiLU.
    np.testing.assert_allclose(got.astype(np.float32), ref, rtol=4e-3, atol=2e-3)
    np.testing.assert_array_equal(got_hist.astype(np.float32), ref_hist)


def test_causal_conv_history_carries_across_steps():
    # Steps of 2 and 5 tokens equal one step of 7 (outputs and history).
    channels, k = 16, 4
    x = _inputs.half_normal(11, 1, (1, 7, channels))
    w = f16(_inputs.normal(11, 2, (channels, k), 0.5))
    hist = _inputs.half_normal(11, 3, (1, channels, k - 1))
    whole, whole_hist = _oracle.causal_conv(x, w, hist, False)
    a, h1 = _oracle.causal_conv(x[:, :2], w, hist, False)
    b, h2 = _oracle.causal_conv(x[:, 2:], w, h1, False)
    np.testing.assert_array_equal(np.concatenate([a, b], 1).view(np.uint16), whole.view(np.uint16))
    np.testing.assert_array_equal(h2.view(np.uint16), whole_hist.view(np.uint16))


def test_l2norm_and_gates_match_transformers():
    x = _inputs.normal(12, 1, (6, 4 * 128))
    got = _oracle.l2norm(x, 128, 1.0 / np.sqrt(128.0))
    ref = (qn.l2norm(torch.from_numpy(x).view(6, 4, 128)) / np.sqrt(128.0)).reshape(6, -1).numpy()
    np.testing.assert_allclose(got, ref, rtol=2e-6, atol=1e-7)

    rows, heads = 9, 8
    a = f16(_inputs.normal(12, 2, (rows, heads), 3.0))
    b = f16(_inputs.normal(12, 3, (rows, heads), 3.0))
    a_log = _inputs.normal(12, 4, (heads,), 1.0)
    dt_bias = _inputs.normal(12, 5, (heads,), 1.0)
    beta, decay = _oracle.delta_gates(a, b, a_log, dt_bias)
    # Qwen3-Next's gated DeltaNet: g = -exp(A_log) softplus(a + dt_bias),
    # beta = sigmoid(b); the reference keeps beta at fp16 precision.
    g = -torch.from_numpy(a_log).exp() * torch.nn.functional.softplus(
        torch.from_numpy(a.astype(np.float32)) + torch.from_numpy(dt_bias))
    np.testing.assert_allclose(decay, g.exp().numpy(), rtol=2e-6, atol=1e-30)
    np.testing.assert_allclose(beta, torch.from_numpy(b.astype(np.float32)).sigmoid().numpy(),
                               rtol=5e-4, atol=1e-6)
