"""GQA parity on the GPU: cacheAppend, prefill (gqaFlashAttention) and
decode (gqaScores + gqaSoftmax), through the C ABI, against the CPU oracle.

Bars: the reference's own known-answer tolerance |a - e| <= 2e-4 + 5e-4|e|
(tests/FlashAttentionTest.mm:80-81) on its two KAT cases, and the acceptance
bar max-abs <= 1e-2, rel-L2 <= 2e-3 against the fp64 dense oracle elsewhere.
Outputs are pre-filled with NaN (as FlashAttentionTest.mm:41 does) so an
unwritten element fails.
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import _inputs
import _oracle
from llminfer_b200 import abi, ops

pytestmark = pytest.mark.gpu

GOLDEN = _oracle.ROOT / "tests" / "golden"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def nan_like(t):
    return torch.full_like(t, float("nan"))


def check_bar(got, expected):
    got = got.float().cpu().numpy() if isinstance(got, torch.Tensor) else got
    assert np.isfinite(got).all(), "unwritten or non-finite outputs"
    max_abs, rel = _inputs.errors(got, expected)
    assert max_abs <= _inputs.MAX_ABS and rel <= _inputs.REL_L2, (max_abs, rel)
    return max_abs, rel


@pytest.mark.parametrize("case", [0, 1])
def test_prefill_known_answers(case):
    kat = np.load(GOLDEN / "gqa_kat.npz")
    T, Hq, Hkv, D, past = (int(x) for x in kat[f"case{case}_shape"])
    q = dev(kat[f"case{case}_q"].view(np.float16).reshape(1, T, Hq, D))
    k = dev(kat[f"case{case}_k"].view(np.float16).reshape(1, past + T, Hkv, D))
    v = dev(kat[f"case{case}_v"].view(np.float16).reshape(1, past + T, Hkv, D))
    out = ops.gqa_prefill(q, k, v, past, out=nan_like(q))
    torch.cuda.synchronize()
    got = out.double().cpu().numpy()
    expected = kat[f"case{case}_expected"].reshape(1, T, Hq, D)
    if D % 16:
        # CUDA-core path, fp32 probabilities: the reference's own tolerance.
        atol = 2e-4
    else:
        # Tensor-core path: P enters the P.V MMA rounded to fp16 (relative
        # error <= 2^-11 per probability), so |error| <= 2^-11 * max|v|
        # (= 9.8e-4 for these inputs, |v| <= 2) on top of the output rounding
        # already covered by the 5e-4|e| term.
        atol = 2.0 ** -11 * np.abs(kat[f"case{case}_v"].view(np.float16)).max() + 2e-5
    assert np.all(np.abs(got - expected) <= atol + 5e-4 * np.abs(expected))


@pytest.mark.parametrize("batch,tokens,past,hq,hkv,d", [
    (1, 128, 0, 16, 4, 256),   # the prefill benchmark config (C1)
    (2, 33, 17, 8, 2, 64),
    (2, 5, 0, 4, 4, 128),
    (3, 70, 130, 16, 4, 256),
    (2, 300, 0, 16, 4, 256),   # many key tiles: running-max rescales, stage reuse
    (2, 40, 10, 8, 1, 256),    # group of 8 (16 tokens per tile)
    (2, 50, 3, 4, 4, 256),     # group of 1 (128 tokens per tile)
    (1, 1100, 200, 16, 4, 256),  # 11 key tiles: K and V rings wrap, odd pair count
    (1, 7, 0, 32, 2, 256),     # group of 16, single partial tile
    (2, 19, 3, 4, 2, 12),      # odd head_dim (CUDA-core path)
    (1, 9, 40, 6, 2, 40),
])
def test_prefill_matches_dense_oracle(batch, tokens, past, hq, hkv, d):
    q, k, v = _inputs.gqa_case(batch, tokens, past, hq, hkv, d, capacity=past + tokens + 3,
                               seed=100 + tokens)
    out = ops.gqa_prefill(dev(q), dev(k), dev(v), past, out=nan_like(dev(q)))
    check_bar(out, _oracle.gqa_dense(q, k, v, past))


@pytest.mark.parametrize("batch,past,hq,hkv,d", [
    (3, 0, 16, 4, 256),
    (3, 15, 16, 4, 256),
    (2, 16, 16, 4, 256),
    (2, 1000, 16, 4, 256),
    (2, 77, 8, 8, 128),
    (2, 300, 16, 2, 256),      # group of 8, 2 kv heads: the whole-row pass of 1 KiB rows
    (2, 300, 8, 1, 256),       # group of 8 on the 8-warp CTA-worker pass (heads 4-7 in the combine)
    (2, 1000, 24, 3, 256),     # group of 8, 3 kv heads: CTA workers over units of 3 heads
    (2, 33, 8, 1, 64),
    (2, 40, 16, 8, 64),        # CTA workers with per-warp pipelines
    (2, 50, 4, 2, 12),         # odd head_dim (CUDA-core path)
    (2, 20, 24, 2, 64),        # group of 12 (CUDA-core path)
    (2, 90, 6, 2, 64),         # group of 3: the merge's scalar path
    (4, 8320, 16, 4, 256),     # C5 decode shape: over 32 partial records per sequence
    (3, 500, 8, 2, 128),       # CTA workers, head_dim 128
    (8, 2000, 4, 1, 256),      # CTA workers, one kv head (a head-sharded rank's shape)
    (2, 8320, 16, 4, 256),     # a sequence-major 8-GPU rank: 74 records per unit, merge in 8 slices
    (2, 3000, 16, 1, 128),     # group of 16: CUDA-core path, keys in groups of four
])
def test_decode_matches_oracles(batch, past, hq, hkv, d):
    q, k, v = _inputs.gqa_case(batch, 1, past, hq, hkv, d, capacity=past + 5, seed=7 + past)
    out = ops.gqa_decode(dev(q), dev(k), dev(v), past, out=nan_like(dev(q)))
    got = out.float().cpu().numpy()
    check_bar(got, _oracle.gqa_dense(q, k, v, past))
    # The reference decode path (fp16 scores and probabilities) agrees too.
    max_abs, rel = _inputs.errors(got, _oracle.gqa_eager_f16(q, k, v, past))
    assert max_abs <= _inputs.MAX_ABS and rel <= 5e-3, (max_abs, rel)


def test_decode_benchmark_shape_reduced_batch():
    # C2 per-sequence shape: past 4096 in a capacity-8192 cache.
    q, k, v = _inputs.gqa_case(6, 1, 4096, 16, 4, 256, capacity=8192, seed=11)
    out = ops.gqa_decode(dev(q), dev(k), dev(v), 4096, out=nan_like(dev(q)))
    check_bar(out, _oracle.gqa_dense(q, k, v, 4096))


def test_decode_and_prefill_agree_on_one_token():
    q, k, v = _inputs.gqa_case(4, 1, 513, 16, 4, 256, seed=12)
    a = ops.gqa_decode(dev(q), dev(k), dev(v), 513)
    b = ops.gqa_prefill(dev(q), dev(k), dev(v), 513)
    max_abs, rel = _inputs.errors(a.float().cpu().numpy(), b.float().cpu().numpy())
    assert max_abs <= 4e-3 and rel <= 2e-3


@pytest.mark.parametrize("batch,past,hq,hkv,d", [
    (3, 700, 16, 4, 256),    # whole rows, 2 KiB (partial_rows<256, 4>)
    (200, 20, 16, 4, 256),   # more sequences than CTAs: a CTA writes several rows
    (2, 515, 8, 2, 256),     # whole rows, 1 KiB (partial_rows<256, 2>)
    (2, 333, 16, 8, 128),    # whole rows (partial_rows<128, 8>)
    (3, 260, 16, 8, 64),     # grouped warps (partial_mma<64>)
    (8, 2000, 4, 1, 256),    # CTA workers (partial_mma_cta<256>)
    (3, 500, 12, 3, 128),    # CTA workers, 3 kv heads
    (2, 100, 8, 2, 96),      # CUDA-core pass: the appends run as their own launches
    (1, 0, 16, 4, 256),      # the new row is the only key
])
@pytest.mark.parametrize("keys_given", [True, False])
def test_decode_append_matches_separate_calls(batch, past, hq, hkv, d, keys_given):
    """llmi_cuda_gqa_decode_append against cacheAppend x2 + gqa_decode: the same
    output bits and the same caches (k_new None: the key row is already written)."""
    q, k, v = _inputs.gqa_case(batch, 1, past, hq, hkv, d, capacity=past + 3, seed=40 + past)
    kn = dev(_inputs.half_normal(1, 41, (batch, 1, hkv, d)))
    vn = dev(_inputs.half_normal(1, 42, (batch, 1, hkv, d)))
    kc_a, vc_a = dev(k), dev(v)
    kc_b, vc_b = kc_a.clone(), vc_a.clone()
    if not keys_given:
        ops.cache_append(kn, kc_b, past)  # written beforehand (as normRope does)
    ops.cache_append(kn, kc_a, past)
    ops.cache_append(vn, vc_a, past)
    want = ops.gqa_decode(dev(q), kc_a, vc_a, past, out=nan_like(dev(q)))
    got = ops.gqa_decode_append(dev(q), kn if keys_given else None, vn, kc_b, vc_b, past,
                                out=nan_like(dev(q)))
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert torch.equal(kc_b.view(torch.int16), kc_a.view(torch.int16))
    assert torch.equal(vc_b.view(torch.int16), vc_a.view(torch.int16))


@pytest.mark.parametrize("batch,past,hq,hkv,d", [
    (2, 8320, 16, 4, 256),   # a sequence-major 8-GPU rank's decode (whole 2 KiB rows)
    (3, 700, 16, 4, 256),
    (2, 515, 8, 2, 256),
    (2, 333, 16, 8, 128),
    (8, 2000, 4, 1, 256),    # CTA workers (the flag does not change this pass)
    (2, 20, 16, 4, 256),     # every worker's first tile holds the newest row
    (1, 0, 16, 4, 256),      # the newest row is the only key
])
def test_settled_decode_matches_unsettled(batch, past, hq, hkv, d):
    """llmi_cuda_gqa_decode_append_ex with LLMI_FLAG_SETTLED: cache rows [0, past)
    are requested before the kernel ahead finishes.  Two layers back to back, as
    a session step issues them, after a synchronisation (what the flag asks
    for): the same output bits and caches as the calls without the flag."""
    layers = []
    for l in range(2):
        q, k, v = _inputs.gqa_case(batch, 1, past, hq, hkv, d, capacity=past + 3,
                                   seed=60 + past + l)
        kn = dev(_inputs.half_normal(1, 61 + l, (batch, 1, hkv, d)))
        vn = dev(_inputs.half_normal(1, 63 + l, (batch, 1, hkv, d)))
        layers.append((dev(q), kn, vn, dev(k), dev(v)))
    results = {}
    for settled in (False, True):
        caches = [(kc.clone(), vc.clone()) for _, _, _, kc, vc in layers]
        outs = [nan_like(q) for q, *_ in layers]
        torch.cuda.synchronize()
        for (q, kn, vn, _, _), (kc, vc), out in zip(layers, caches, outs):
            ops.gqa_decode_append(q, kn, vn, kc, vc, past, out=out, settled=settled)
        torch.cuda.synchronize()
        results[settled] = (outs, caches)
    for a, b in zip(results[False][0], results[True][0]):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    for (ka, va), (kb, vb) in zip(results[False][1], results[True][1]):
        assert torch.equal(ka.view(torch.int16), kb.view(torch.int16))
        assert torch.equal(va.view(torch.int16), vb.view(torch.int16))
    check_bar(results[True][0][0], _oracle.gqa_dense(*(t.cpu().numpy() for t in (
        layers[0][0], results[True][1][0][0], results[True][1][0][1])), past))


def test_decode_rejects_small_workspace():
    q, k, v = _inputs.gqa_case(2, 1, 100, 16, 4, 256, seed=13)
    small = torch.empty(256, dtype=torch.uint8, device="cuda")
    with pytest.raises(abi.LlmiError) as err:
        ops.gqa_decode(dev(q), dev(k), dev(v), 100, workspace=small)
    assert err.value.status == abi.LLMI_WORKSPACE_TOO_SMALL


@pytest.mark.parametrize("tokens,past,hkv,d", [(1, 4096, 4, 256), (17, 5, 2, 64), (3, 0, 1, 12)])
def test_cache_append_is_exact(tokens, past, hkv, d):
    batch, cap = 3, past + tokens + 2
    cache = _inputs.half_normal(1, 50, (batch, cap, hkv, d))
    rows = _inputs.half_normal(1, 51, (batch, tokens, hkv, d))
    got = dev(cache)
    ops.cache_append(dev(rows), got, past)
    expected = cache.copy()
    expected[:, past:past + tokens] = rows
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint16), expected.view(np.uint16))


def test_poll_error_is_clean_after_work():
    q, k, v = _inputs.gqa_case(2, 1, 64, 16, 4, 256, seed=14)
    ops.gqa_decode(dev(q), dev(k), dev(v), 64)
    ops.poll_error()


def test_single_cta_prefill_kernel():
    """The single-CTA tensor-core prefill (LLMI_PREFILL_CTA_PAIRS=0, read
    once per process) passes the same prefill parity cases in a child."""
    env = dict(os.environ, LLMI_PREFILL_CTA_PAIRS="0")
    here = os.path.dirname(os.path.abspath(__file__))
    run = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", "-m", "gpu",
         "-k", "prefill and not single_cta", os.path.join(here, "test_gqa_gpu.py")],
        env=env, capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-3000:]
