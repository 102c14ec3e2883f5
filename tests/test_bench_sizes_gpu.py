"""Parity at the sizes the benchmark runs, through the C ABI.

Every benchmarked configuration is checked against the CPU oracle at its own
size (work splits, chunk counts and tile counts differ from the reduced
cases in the other test files):
  C2  GQA decode, 64 sequences, past 4096, capacity 8192 (the real split points);
  C3  DeltaNet prefill, 4 sequences x 4096 tokens = 64 chunks, outputs and
      final state (Graph.metal:146-170, Reference.metal:182-197);
  C5  the hybrid stack's DeltaNet layer length, 8192 tokens = 128 chunks;
  C4  DeltaNet step, 256 sequences;
  C5  GQA prefill, 16 sequences x 8192 tokens, on sampled rows spread over
      the last query tiles, against the fp64 dense check
      (tests/FlashAttentionTest.mm:53-85) evaluated on those rows only.
Bar: max-abs <= 1e-2 and rel-L2 <= 2e-3; outputs are prefilled with NaN.
Each test prints its measured errors (pytest -s shows them).
"""
import numpy as np
import pytest
import torch

import _inputs
import _oracle
from llminfer_b200 import ops

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def report(name, got, want):
    assert np.isfinite(got).all(), f"{name}: unwritten or non-finite outputs"
    max_abs, rel = _inputs.errors(got, want)
    print(f"\nPARITY {name}: max-abs {max_abs:.3e} rel-L2 {rel:.3e}")
    assert max_abs <= _inputs.MAX_ABS and rel <= _inputs.REL_L2, (name, max_abs, rel)


def run_delta(case, workspace):
    state = dev(case["state"])
    out = torch.full(case["v"].shape, float("nan"), dtype=torch.float16, device="cuda")
    ops.delta_update(dev(case["q"]), dev(case["k"]), dev(case["v"]), dev(case["beta"]),
                     dev(case["decay"]), state, out=out, workspace=workspace)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), state.cpu().numpy()


@pytest.mark.parametrize("name,batch,tokens,std", [
    ("C3 DeltaNet prefill B=4 T=4096", 4, 4096, 0.0),
    ("C5 DeltaNet layer length B=1 T=8192", 1, 8192, 0.0),
    ("C4 DeltaNet step B=256", 256, 1, 0.02),
])
def test_delta_at_benchmark_size(name, batch, tokens, std):
    case = _inputs.delta_case(batch, tokens, 16, 128, 32, 128, state_std=std, seed=41)
    want_out, want_state = _oracle.delta_update(case["q"], case["k"], case["v"], case["beta"],
                                                case["decay"], case["state"])
    # Both entry points: with scratch (chunk systems solved in parallel, the
    # form the benchmark runs) and without (one kernel per head).
    forms = (("", None), (" [no scratch]", False)) if tokens > 1 else (("", None),)
    for tag, ws in forms:
        got_out, got_state = run_delta(case, ws)
        report(name + tag + " output", got_out, want_out)
        report(name + tag + " state", got_state, want_state)


def test_decode_c2_full_batch():
    q, k, v = _inputs.gqa_case(64, 1, 4096, 16, 4, 256, capacity=8192, seed=43)
    out = ops.gqa_decode(dev(q), dev(k), dev(v), 4096,
                         out=torch.full(q.shape, float("nan"), dtype=torch.float16,
                                        device="cuda"))
    got = out.float().cpu().numpy()
    report("C2 GQA decode B=64 past 4096", got, _oracle.gqa_dense(q, k, v, 4096))


def test_prefill_c5_shape_sampled_rows():
    B, T, Hq, Hkv, D = 16, 8192, 16, 4, 256
    g = torch.Generator(device="cuda").manual_seed(45)
    q = torch.randn(B, T, Hq, D, generator=g, device="cuda").half()
    k = torch.randn(B, T, Hkv, D, generator=g, device="cuda").half()
    v = torch.randn(B, T, Hkv, D, generator=g, device="cuda").half()
    out = ops.gqa_prefill(q, k, v, 0, out=torch.full_like(q, float("nan")))
    torch.cuda.synchronize()
    assert torch.isfinite(out).all().item(), "unwritten or non-finite outputs"
    # Rows spread over the sequences and heads, mostly in the last query
    # tiles (the longest rows: 64 key tiles), plus the first and a middle one.
    rng = np.random.default_rng(45)
    tokens = np.concatenate([T - 1 - rng.integers(0, 512, 40), [0, 127, 4095, 4096, 8064]])
    seqs = rng.integers(0, B, tokens.size)
    heads = rng.integers(0, Hq, tokens.size)
    got, want = [], []
    for s in np.unique(seqs):
        sel = seqs == s
        ks = k[s].cpu().numpy()
        vs = v[s].cpu().numpy()
        rows = q[s].cpu().numpy()[tokens[sel], heads[sel]]
        want.append(_oracle.gqa_dense_rows(rows, ks, vs, 0, T, Hq, tokens[sel], heads[sel]))
        got.append(out[s].float().cpu().numpy()[tokens[sel], heads[sel]])
    report("C5 GQA prefill B=16 T=8192 (45 sampled rows)", np.concatenate(got),
           np.concatenate(want))
