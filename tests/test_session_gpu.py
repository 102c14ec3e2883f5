"""The attention-stack session on the GPU: state ownership, past/capacity
rules, --plan names and parity of a chunked run against the oracle, mirroring
tests/MetalReferenceTest.py (test_long_attention: partial tiles, nonzero
past and the switch to decode; partition invariance).
"""
import numpy as np
import pytest
import torch

import _inputs
import _oracle
from llminfer_b200 import abi, ops

pytestmark = pytest.mark.gpu

KINDS = [abi.LAYER_DELTANET, abi.LAYER_DELTANET, abi.LAYER_DELTANET, abi.LAYER_GQA]
SHAPE = dict(query_heads=8, kv_heads=2, head_dim=256, key_heads=2, key_dim=128,
             value_heads=4, value_dim=128)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


class HostModel:
    """Oracle-side copy of the session: caches and recurrent states."""

    def __init__(self, batch, capacity):
        s = SHAPE
        self.keys = np.zeros((batch, capacity, s["kv_heads"], s["head_dim"]), np.float16)
        self.values = np.zeros_like(self.keys)
        self.states = [np.zeros((batch, s["value_heads"], s["key_dim"], s["value_dim"]), np.float32)
                       for _ in KINDS]
        self.past = 0


def make_inputs(batch, tokens, layer, seed):
    s = SHAPE
    if KINDS[layer] == abi.LAYER_GQA:
        q = _inputs.half_normal(seed, 100 + layer, (batch, tokens, s["query_heads"], s["head_dim"]))
        k = _inputs.half_normal(seed, 200 + layer, (batch, tokens, s["kv_heads"], s["head_dim"]))
        v = _inputs.half_normal(seed, 300 + layer, (batch, tokens, s["kv_heads"], s["head_dim"]))
        return dict(q=q, k=k, v=v)
    return _inputs.delta_case(batch, tokens, s["key_heads"], s["key_dim"], s["value_heads"],
                              s["value_dim"], seed=seed * 7 + layer)


def to_layer(x):
    out_shape = x["q"].shape if "beta" not in x else x["v"].shape
    out = torch.full(out_shape, float("nan"), dtype=torch.float16, device="cuda")
    if "beta" in x:
        return ops.LayerTensors(q=dev(x["q"]), k=dev(x["k"]), v=dev(x["v"]), out=out,
                                beta=dev(x["beta"]), decay=dev(x["decay"]))
    return ops.LayerTensors(q=dev(x["q"]), k=dev(x["k"]), v=dev(x["v"]), out=out)


def oracle_step(host, inputs, tokens):
    outs = []
    for layer, x in enumerate(inputs):
        if KINDS[layer] == abi.LAYER_GQA:
            host.keys[:, host.past:host.past + tokens] = x["k"]
            host.values[:, host.past:host.past + tokens] = x["v"]
            outs.append(_oracle.gqa_dense(x["q"], host.keys, host.values, host.past))
        else:
            o, host.states[layer] = _oracle.delta_update(x["q"], x["k"], x["v"], x["beta"],
                                                         x["decay"], host.states[layer])
            outs.append(o)
    host.past += tokens
    return outs


def test_chunked_session_matches_oracle_and_reports_plan():
    batch, capacity = 2, 64
    session = ops.AttentionSession(KINDS, batch, capacity, **SHAPE)
    host = HostModel(batch, capacity)
    for step, tokens in enumerate([17, 5, 1, 1]):
        inputs = [make_inputs(batch, tokens, l, seed=1000 + step) for l in range(len(KINDS))]
        layers = [to_layer(x) for x in inputs]
        session.step(tokens, layers, trace_plan=True)
        expected = oracle_step(host, inputs, tokens)
        for layer, (got, want) in enumerate(zip(layers, expected)):
            g = got.out.float().cpu().numpy()
            assert np.isfinite(g).all(), (step, layer)
            max_abs, rel = _inputs.errors(g, want)
            assert max_abs <= _inputs.MAX_ABS and rel <= _inputs.REL_L2, (step, layer, max_abs, rel)
        kernels = {d["kernel"] for d in session.plan()}
        assert ("gqaFlashAttention" in kernels) == (tokens > 1)
        assert ("gqaSoftmax" in kernels) != (tokens > 1)
        assert ("gqaScores" in kernels) != (tokens > 1)
        assert session.past == host.past
    keys = session.read_state(3, abi.STATE_KEYS).cpu().numpy()
    np.testing.assert_array_equal(keys.view(np.uint16), host.keys.view(np.uint16))
    state = session.read_state(0, abi.STATE_RECURRENT).cpu().numpy()
    max_abs, rel = _inputs.errors(state, host.states[0])
    assert max_abs <= _inputs.MAX_ABS and rel <= _inputs.REL_L2
    session.reset()
    assert session.past == 0 and not session.invalid
    assert not session.read_state(0, abi.STATE_RECURRENT).any()
    session.close()


def test_capacity_is_enforced_before_launch():
    session = ops.AttentionSession(KINDS, 1, 8, **SHAPE)
    inputs = [to_layer(make_inputs(1, 6, l, seed=5)) for l in range(len(KINDS))]
    session.step(6, inputs)
    before = session.read_state(3, abi.STATE_KEYS).clone()
    too_many = [to_layer(make_inputs(1, 3, l, seed=6)) for l in range(len(KINDS))]
    with pytest.raises(abi.LlmiError) as err:
        session.step(3, too_many)
    assert err.value.status == abi.LLMI_CAPACITY_EXCEEDED
    assert session.past == 6 and not session.invalid
    assert torch.equal(session.read_state(3, abi.STATE_KEYS), before)
    session.close()


def test_partition_invariance():
    batch, capacity = 1, 32
    full_inputs = [make_inputs(batch, 12, l, seed=77) for l in range(len(KINDS))]
    a = ops.AttentionSession(KINDS, batch, capacity, **SHAPE)
    full = [to_layer(x) for x in full_inputs]
    a.step(12, full)
    b = ops.AttentionSession(KINDS, batch, capacity, **SHAPE)
    outs = []
    for lo, hi in [(0, 5), (5, 12)]:
        part = [to_layer({n: v[:, lo:hi] if n != "state" else v for n, v in x.items()})
                for x in full_inputs]
        b.step(hi - lo, part)
        outs.append(part)
    for layer in range(len(KINDS)):
        joined = torch.cat([outs[0][layer].out, outs[1][layer].out], dim=1)
        torch.testing.assert_close(joined.float(), full[layer].out.float(), atol=1e-3, rtol=1e-3)
        if KINDS[layer] == abi.LAYER_DELTANET:
            torch.testing.assert_close(b.read_state(layer, abi.STATE_RECURRENT),
                                       a.read_state(layer, abi.STATE_RECURRENT),
                                       atol=1e-5, rtol=1e-5)
    a.close()
    b.close()
