"""Producers of the path's operands on the GPU, through the C ABI, against the
CPU oracle (itself pinned to transformers' Qwen3-Next code in
test_producers.py).

Bar: fp16 outputs within 2 fp16 ulps (RoPE outputs: one fp16 ulp at unit
scale), with at most 1 % of elements differing at all; fp32 q/k within
4e-6 relative, decay within 2e-5.  The kernels keep the reference's rounding points; what may
differ is the order of row sums (warp trees) and the last bit of expf,
powf or cosf.
"""
import numpy as np
import pytest
import torch

import _inputs
import _oracle
from llminfer_b200 import abi, ops

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def ulps(a, b):
    a = np.asarray(a, np.float16).astype(np.float32)
    b = np.asarray(b, np.float16).astype(np.float32)
    scale = np.maximum(np.abs(a), np.abs(b))
    ulp = np.where(scale < 2.0 ** -14, 2.0 ** -24,
                   2.0 ** (np.floor(np.log2(np.maximum(scale, 1e-30))) - 10))
    return np.abs(a - b) / ulp


def check_f16(got, expected, max_ulps=2, max_frac=0.01, unit_scale=False):
    """Within max_ulps of the expected value (or, with unit_scale, within
    2^-9 * max(1, |expected|): RoPE phases at large positions can move cos/sin
    by one fp16 ulp, which a small output shows as many of its own ulps),
    and at most max_frac of the elements differing at all."""
    got = got.cpu().numpy() if isinstance(got, torch.Tensor) else got
    assert np.isfinite(got.astype(np.float32)).all()
    u = ulps(got, expected)
    assert (u > 0).mean() <= max_frac, (u > 0).mean()
    if unit_scale:
        e = np.asarray(expected, np.float32)
        d = np.abs(np.asarray(got, np.float32) - e)
        assert np.all(d <= 2.0 ** -9 * np.maximum(1.0, np.abs(e))), d.max()
    else:
        assert u.max() <= max_ulps, u.max()


@pytest.mark.parametrize("batch,tokens,past,heads,d,rot,stride", [
    (1, 128, 0, 16, 256, 64, 512),    # q of the C1 shape, sliced from [q | gate]
    (2, 7, 4090, 4, 256, 64, 256),    # k rows at large positions
    (3, 5, 11, 3, 64, 32, 64),
    (1, 9, 2, 2, 40, 16, 40),         # head_dim not a multiple of 8 (scalar path)
])
def test_norm_rope(batch, tokens, past, heads, d, rot, stride):
    x = _inputs.half_normal(20 + tokens, 1, (batch, tokens, heads, stride))
    w = _inputs.normal(20 + tokens, 2, (d,), 0.1)
    expected = _oracle.norm_rope(x, w, past, rot, 10_000_000.0, head_dim=d)
    got = ops.norm_rope(dev(x), dev(w), past, rot, 10_000_000.0, head_dim=d)
    check_f16(got, expected, unit_scale=True)


def test_norm_rope_writes_key_cache_rows():
    # k rows of a step straight into the cache at row `past` (cacheAppend).
    batch, tokens, past, heads, d, cap = 2, 6, 33, 4, 256, 48
    x = _inputs.half_normal(31, 1, (batch, tokens, heads, d))
    w = _inputs.normal(31, 2, (d,), 0.1)
    cache = _inputs.half_normal(31, 3, (batch, cap, heads, d))
    expected = _oracle.norm_rope(x, w, past, 64, 10_000_000.0, output=cache, output_start=past)
    got = dev(cache)
    ops.norm_rope(dev(x), dev(w), past, 64, 10_000_000.0, out=got, output_start=past)
    got = got.cpu().numpy()
    np.testing.assert_array_equal(got[:, :past].view(np.uint16), cache[:, :past].view(np.uint16))
    np.testing.assert_array_equal(got[:, past + tokens:].view(np.uint16),
                                  cache[:, past + tokens:].view(np.uint16))
    check_f16(got[:, past:past + tokens], expected[:, past:past + tokens], unit_scale=True)


def test_partial_rope():
    x = _inputs.half_normal(32, 1, (2, 10, 4, 128))
    expected = _oracle.norm_rope(x, None, 70, 64, 10000.0)
    check_f16(ops.norm_rope(dev(x), None, 70, 64, 10000.0), expected, unit_scale=True)


@pytest.mark.parametrize("batch,tokens,channels,k,silu", [
    (2, 1, 96, 4, True), (1, 2, 64, 4, False), (3, 37, 200, 4, True), (2, 9, 33, 3, True)])
def test_causal_conv(batch, tokens, channels, k, silu):
    x = _inputs.half_normal(40 + tokens, 1, (batch, tokens, channels))
    w = _inputs.normal(40 + tokens, 2, (channels, k), 0.5).astype(np.float16)
    hist = _inputs.half_normal(40 + tokens, 3, (batch, channels, k - 1))
    expected, exp_hist = _oracle.causal_conv(x, w, hist, silu)
    h = dev(hist)
    got = ops.causal_conv(dev(x), dev(w), h, silu)
    check_f16(got, expected)
    np.testing.assert_array_equal(h.cpu().numpy().view(np.uint16), exp_hist.view(np.uint16))


@pytest.mark.parametrize("batch,tokens,hk,hv", [
    (2, 1, 4, 8), (1, 3, 4, 8), (2, 70, 4, 8),
    (2, 40, 2, 5),   # 9 heads: the second group of 8 holds one
    (2, 2000, 16, 32),  # the C5 heads: more (sequence, tile, head) items than resident warps
])
def test_delta_prepare(batch, tokens, hk, hv):
    dk, dv, kern = 128, 128, 4
    width = 2 * hk * dk + hv * dv
    qkv = _inputs.half_normal(50 + tokens, 1, (batch, tokens, width))
    w = _inputs.normal(50 + tokens, 2, (width, kern), 0.5).astype(np.float16)
    hist = _inputs.half_normal(50 + tokens, 3, (batch, width, kern - 1))
    eq, ek, ev, eh = _oracle.delta_prepare(qkv, w, hist, hk, dk, hv, dv)
    h = dev(hist)
    q, k, v = ops.delta_prepare(dev(qkv), dev(w), h, hk, dk, hv, dv)
    np.testing.assert_allclose(q.cpu().numpy(), eq, rtol=4e-6, atol=1e-7)
    np.testing.assert_allclose(k.cpu().numpy(), ek, rtol=4e-6, atol=1e-7)
    check_f16(v, ev)
    np.testing.assert_array_equal(h.cpu().numpy().view(np.uint16), eh.view(np.uint16))


def test_delta_prepare_silu_table_matches_computed_silu():
    # The tiled deltaPrepare takes half(silu(half(acc))) from a per-device
    # fp16 table (copied into shared memory); the element-wise causalConv
    # computes it.  The v channels of
    # both must agree bit for bit over a wide range of conv outputs.
    batch, tokens, hk, dk, hv, dv, kern = 2, 50, 2, 128, 4, 128, 4
    width = 2 * hk * dk + hv * dv
    qkv = (_inputs.half_normal(80, 1, (batch, tokens, width)).astype(np.float32) * 8).astype(np.float16)
    w = _inputs.normal(80, 2, (width, kern), 1.0).astype(np.float16)
    hist = _inputs.half_normal(80, 3, (batch, width, kern - 1))
    _, _, v = ops.delta_prepare(dev(qkv), dev(w), dev(hist), hk, dk, hv, dv)
    conv = ops.causal_conv(dev(qkv), dev(w), dev(hist), True)
    np.testing.assert_array_equal(v.cpu().numpy().view(np.uint16),
                                  conv[..., 2 * hk * dk:].cpu().numpy().view(np.uint16))


def test_delta_prepare_feeds_delta_update():
    # prepare -> gates -> graphDeltaUpdate on the GPU equals the oracle chain.
    batch, tokens, hk, dk, hv, dv, kern = 1, 20, 2, 128, 4, 128, 4
    width = 2 * hk * dk + hv * dv
    qkv = _inputs.half_normal(60, 1, (batch, tokens, width))
    w = _inputs.normal(60, 2, (width, kern), 0.5).astype(np.float16)
    hist = np.zeros((batch, width, kern - 1), np.float16)
    a = _inputs.normal(60, 3, (batch, tokens, hv), 2.0).astype(np.float16)
    b = _inputs.normal(60, 4, (batch, tokens, hv), 2.0).astype(np.float16)
    a_log = _inputs.normal(60, 5, (hv,), 0.5)
    dt_bias = _inputs.normal(60, 6, (hv,), 0.5)
    state = np.zeros((batch, hv, dk, dv), np.float32)

    eq, ek, ev, _ = _oracle.delta_prepare(qkv, w, hist, hk, dk, hv, dv)
    ebeta, edecay = _oracle.delta_gates(a.reshape(-1, hv), b.reshape(-1, hv), a_log, dt_bias)
    eout, _ = _oracle.delta_update(eq, ek, ev, ebeta.reshape(batch, tokens, hv),
                                   edecay.reshape(batch, tokens, hv), state)

    q, k, v = ops.delta_prepare(dev(qkv), dev(w), dev(hist), hk, dk, hv, dv)
    beta, decay = ops.delta_gates(dev(a), dev(b), dev(a_log), dev(dt_bias))
    out = ops.delta_update(q, k, v, beta, decay, dev(state))
    max_abs, rel = _inputs.errors(out.float().cpu().numpy(), eout.astype(np.float32))
    assert max_abs <= _inputs.MAX_ABS and rel <= _inputs.REL_L2, (max_abs, rel)


def test_l2_norm_and_gates():
    x = _inputs.half_normal(70, 1, (33, 4 * 128))
    expected = _oracle.l2norm(x.astype(np.float32), 128, 1.0 / np.sqrt(128.0))
    got = ops.l2_norm(dev(x), 128, 1.0 / np.sqrt(128.0))
    np.testing.assert_allclose(got.cpu().numpy(), expected, rtol=4e-6, atol=1e-7)

    a = _inputs.normal(70, 2, (17, 32), 3.0).astype(np.float16)
    b = _inputs.normal(70, 3, (17, 32), 3.0).astype(np.float16)
    a_log = _inputs.normal(70, 4, (32,), 1.0)
    dt_bias = _inputs.normal(70, 5, (32,), 1.0)
    ebeta, edecay = _oracle.delta_gates(a, b, a_log, dt_bias)
    beta, decay = ops.delta_gates(dev(a), dev(b), dev(a_log), dev(dt_bias))
    # beta is fp16-valued (one fp16 ulp if expf's last bit moves a rounding);
    # decay = exp(x) carries x's relative error times |x| (|x| up to ~100 here).
    np.testing.assert_allclose(beta.cpu().numpy(), ebeta, rtol=2.0 ** -10, atol=0)
    np.testing.assert_allclose(decay.cpu().numpy(), edecay, rtol=2e-5, atol=0)


def test_producer_argument_errors():
    x = torch.zeros(1, 2, 2, 2048, dtype=torch.float16, device="cuda")
    with pytest.raises(abi.LlmiError) as err:
        ops.norm_rope(x, torch.zeros(2048, device="cuda"), 0, 64, 1e4)
    assert err.value.status == abi.LLMI_UNSUPPORTED
    qkv = torch.zeros(1, 2, 100, dtype=torch.float16, device="cuda")
    with pytest.raises(abi.LlmiError) as err:
        ops.delta_prepare(qkv, torch.zeros(100, 4, dtype=torch.float16, device="cuda"),
                          torch.zeros(1, 100, 3, dtype=torch.float16, device="cuda"), 1, 16, 1, 16)
    assert err.value.status == abi.LLMI_INVALID_ARGUMENT
