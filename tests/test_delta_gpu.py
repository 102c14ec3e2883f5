"""Gated-DeltaNet parity on the GPU (graphDeltaUpdate through the C ABI)
against the token-sequential CPU oracle restated from Graph.metal:146-170 /
Reference.metal:182-197.  Bar: max-abs <= 1e-2 and rel-L2 <= 2e-3 on the
fp16 outputs and on the updated fp32 state.
"""
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


# The two entry points: llmi_cuda_delta_update_ws (chunk systems solved for
# every chunk at once, then the state pass) and llmi_cuda_delta_update (one
# kernel per head that solves each chunk's system in order, no scratch).
FORMS = {"presolved": None, "fused": False}


def run(case, form="presolved"):
    state = dev(case["state"])
    out = torch.full(case["v"].shape, float("nan"), dtype=torch.float16, device="cuda")
    ops.delta_update(dev(case["q"]), dev(case["k"]), dev(case["v"]), dev(case["beta"]),
                     dev(case["decay"]), state, out=out, workspace=FORMS[form])
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), state.cpu().numpy()


def check(case, got_out, got_state):
    want_out, want_state = _oracle.delta_update(case["q"], case["k"], case["v"], case["beta"],
                                                case["decay"], case["state"])
    assert np.isfinite(got_out).all()
    for got, want in ((got_out, want_out), (got_state, want_state)):
        max_abs, rel = _inputs.errors(got, want)
        assert max_abs <= _inputs.MAX_ABS and rel <= _inputs.REL_L2, (max_abs, rel)


@pytest.mark.parametrize("batch,tokens,hk,dk,hv,dv,std", [
    (16, 1, 16, 128, 32, 128, 0.02),  # the recurrent-step config (C4), fewer sequences
    (16, 3, 16, 128, 32, 128, 0.02),  # 32-column items, four per CTA, a few tokens
    (8, 2, 8, 64, 32, 128, 0.02),     # the same with dk 64, two items per CTA
    (20, 1, 16, 128, 32, 128, 0.02),  # enough (sequence, head) pairs for 128-column CTAs
    (24, 3, 8, 64, 32, 128, 0.02),    # the same, dk 64, a few tokens
    (3, 1, 16, 128, 32, 128, 0.0),
    (2, 1, 4, 64, 8, 128, 0.02),
    (2, 37, 2, 128, 4, 128, 0.02),    # one partial chunk (chunked kernel)
    (2, 200, 2, 128, 4, 128, 0.02),   # several chunks, last one partial
    (1, 64, 1, 128, 2, 128, 0.0),     # exactly one chunk
    (3, 15, 2, 128, 4, 128, 0.02),    # below the chunked threshold
    (2, 3, 2, 7, 4, 5, 0.02),         # odd dims (generic kernel)
    (1, 130, 2, 16, 4, 8, 0.02),
])
@pytest.mark.parametrize("form", sorted(FORMS))
def test_delta_matches_oracle(batch, tokens, hk, dk, hv, dv, std, form):
    case = _inputs.delta_case(batch, tokens, hk, dk, hv, dv, state_std=std, seed=31 + tokens)
    check(case, *run(case, form))


@pytest.mark.parametrize("form", sorted(FORMS))
def test_delta_prefill_config_reduced(form):
    # C3 per-sequence shape (16 key heads, 32 value heads, 128 x 128), shorter.
    case = _inputs.delta_case(1, 256, 16, 128, 32, 128, seed=33)
    check(case, *run(case, form))


@pytest.mark.parametrize("hk,hv", [(4, 4), (2, 8), (1, 3), (1, 6)])
def test_presolved_groups(hk, hv):
    # Key heads shared by 1, 4, 3 and 6 value heads: the solve pass walks the
    # value heads of its key head (up to 4 with their gates derived up front,
    # more one at a time); ragged last chunk, a decay of exactly 0.
    case = _inputs.delta_case(2, 150, hk, 128, hv, 128, state_std=0.02, seed=hv)
    case["decay"][1, 70, 0] = 0.0
    check(case, *run(case, "presolved"))
    check(case, *run(case, "fused"))


def test_presolved_rejects_small_workspace():
    case = _inputs.delta_case(1, 64, 1, 128, 2, 128, seed=3)
    small = torch.empty(8192, dtype=torch.uint8, device="cuda")  # needs 2 x 8 KB
    out = torch.full(case["v"].shape, float("nan"), dtype=torch.float16, device="cuda")
    with pytest.raises(abi.LlmiError) as err:
        ops.delta_update(dev(case["q"]), dev(case["k"]), dev(case["v"]), dev(case["beta"]),
                         dev(case["decay"]), dev(case["state"]), out=out, workspace=small)
    assert err.value.status == abi.LLMI_WORKSPACE_TOO_SMALL
    torch.cuda.synchronize()
    assert torch.isnan(out).all()


@pytest.mark.parametrize("batch,tokens,hk,dk", [
    (2, 1, 16, 128),    # a sequence-major 8-GPU rank's step: 32-column CTAs
    (16, 1, 16, 128),   # the 1-GPU stack's step
    (3, 5, 16, 128),    # a few tokens
    (8, 2, 8, 64),      # dk 64
    (20, 1, 16, 128),   # 128-column CTAs (the flag does not change them)
])
def test_settled_update_matches_unsettled(batch, tokens, hk, dk):
    """llmi_cuda_delta_update_ws_ex with LLMI_FLAG_SETTLED: the state is loaded
    before the kernel ahead finishes.  Three layers' states back to back, as a
    session step issues them, after a synchronisation: the same output and
    state bits as the calls without the flag."""
    cases = [_inputs.delta_case(batch, tokens, hk, dk, 32, 128, state_std=0.02, seed=70 + l)
             for l in range(3)]
    ws = torch.empty(16, dtype=torch.uint8, device="cuda")
    results = {}
    for settled in (False, True):
        states = [dev(c["state"]) for c in cases]
        outs = [torch.full(c["v"].shape, float("nan"), dtype=torch.float16, device="cuda")
                for c in cases]
        args = [[dev(c[n]) for n in ("q", "k", "v", "beta", "decay")] for c in cases]
        torch.cuda.synchronize()
        for a, st, out in zip(args, states, outs):
            ops.delta_update(*a, st, out=out, workspace=ws, settled=settled)
        torch.cuda.synchronize()
        results[settled] = (outs, states)
    for a, b in zip(results[False][0], results[True][0]):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    for a, b in zip(results[False][1], results[True][1]):
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    check(cases[0], results[True][0][0].float().cpu().numpy(), results[True][1][0].cpu().numpy())


@pytest.mark.parametrize("form", sorted(FORMS))
def test_delta_matches_transformers_fixture(form):
    d = np.load(GOLDEN / "delta_xcheck.npz")
    case = dict(q=d["q"], k=d["k"], v=d["v"].view(np.float16), beta=d["beta"],
                decay=d["decay"], state=d["state"])
    out, state = run(case, form)
    max_abs, rel = _inputs.errors(out, d["recurrent_out"])
    assert max_abs <= _inputs.MAX_ABS and rel <= _inputs.REL_L2, (max_abs, rel)
    max_abs, rel = _inputs.errors(state, d["recurrent_state"])
    assert max_abs <= _inputs.MAX_ABS and rel <= _inputs.REL_L2, (max_abs, rel)


@pytest.mark.parametrize("total,cut", [(12, 5), (40, 13), (200, 131)])
def test_delta_chunking_is_invariant(total, cut):
    # One call over all tokens vs two calls.  Short calls run the
    # token-sequential kernel and long ones the chunked form, whose products
    # take fp16 operands, so the two agree to fp16 operand rounding; calls on
    # the same kernel agree to fp32 rounding.
    case = _inputs.delta_case(2, total, 2, 128, 4, 128, state_std=0.02, seed=35 + total)
    full_out, full_state = run(case)
    first = {n: (a[:, :cut] if n != "state" else a) for n, a in case.items()}
    out1, s1 = run(first)
    second = {n: (a[:, cut:] if n != "state" else s1) for n, a in case.items()}
    out2, s2 = run(second)
    tol = 1e-5 if total < 16 else 2e-3
    np.testing.assert_allclose(np.concatenate([out1, out2], axis=1), full_out, atol=tol, rtol=tol)
    np.testing.assert_allclose(s2, full_state, atol=tol, rtol=tol)
