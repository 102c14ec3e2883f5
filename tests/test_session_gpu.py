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


def test_decode_steps_agree_however_they_are_issued():
    # The session passes LLMI_FLAG_SETTLED to its decode-path calls only when
    # its earlier steps are known complete: after a synchronising step, and
    # for the first step of each stream capture, not for a step enqueued
    # behind an unsynchronised one.  The three ways of issuing the same decode
    # steps must give the same bits (outputs, caches and states).
    batch, capacity, prefill, steps = 2, 64, 20, 4
    pre = [make_inputs(batch, prefill, l, seed=90) for l in range(len(KINDS))]
    dec = [[make_inputs(batch, 1, l, seed=91 + i) for l in range(len(KINDS))]
           for i in range(steps)]
    results = {}
    for mode in ("step", "enqueue", "graphs"):
        session = ops.AttentionSession(KINDS, batch, capacity, **SHAPE)
        session.step(prefill, [to_layer(x) for x in pre])
        layers = [[to_layer(x) for x in d] for d in dec]
        torch.cuda.synchronize()
        if mode == "step":
            for step_layers in layers:
                session.step(1, step_layers)
        elif mode == "enqueue":
            for step_layers in layers:
                session.enqueue(1, step_layers)
            session.sync()
        else:
            graphs = []
            for step_layers in layers:
                table = session.operand_table(step_layers)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=session.stream):
                    session.enqueue(1, table)
                graphs.append((g, table))
            for g, _ in graphs:
                g.replay()
            torch.cuda.synchronize()
            session.sync()
            del graphs
        assert session.past == prefill + steps
        outs = [x.out.clone() for step_layers in layers for x in step_layers]
        states = [session.read_state(l, abi.STATE_RECURRENT if k == abi.LAYER_DELTANET
                                     else abi.STATE_KEYS).clone() for l, k in enumerate(KINDS)]
        results[mode] = (outs, states)
        session.close()
    for mode in ("enqueue", "graphs"):
        for a, b in zip(results["step"][0] + results["step"][1],
                        results[mode][0] + results[mode][1]):
            assert torch.equal(a.view(torch.uint8), b.view(torch.uint8)), mode


PRODUCER_KINDS = [abi.LAYER_DELTANET, abi.LAYER_GQA]


def projection_inputs(batch, tokens, seed):
    """Projection outputs and weights of one step for PRODUCER_KINDS."""
    s = SHAPE
    width = 2 * s["key_heads"] * s["key_dim"] + s["value_heads"] * s["value_dim"]
    hv = s["value_heads"]
    delta = dict(
        qkv=dev(_inputs.half_normal(seed, 1, (batch, tokens, width))),
        a=dev(_inputs.normal(seed, 2, (batch, tokens, hv), 2.0).astype(np.float16)),
        b=dev(_inputs.normal(seed, 3, (batch, tokens, hv), 2.0).astype(np.float16)))
    gqa = dict(
        qg=dev(_inputs.half_normal(seed, 4, (batch, tokens, s["query_heads"], 2 * s["head_dim"]))),
        k=dev(_inputs.half_normal(seed, 5, (batch, tokens, s["kv_heads"], s["head_dim"]))),
        v=dev(_inputs.half_normal(seed, 6, (batch, tokens, s["kv_heads"], s["head_dim"]))))
    return delta, gqa


def test_step_projections_equals_the_composed_producers_and_ops():
    # The session's producer path runs the same kernels as composing the ops
    # by hand (norm_rope into the cache, cache_append of v, the attention;
    # delta_prepare over the conv history, delta_gates, delta_update), so
    # outputs and every state agree bit for bit: a prefill, a decode step and
    # a short multi-token step.
    s = SHAPE
    batch, capacity, rot, theta, conv = 2, 64, 64, 10_000_000.0, 4
    width = 2 * s["key_heads"] * s["key_dim"] + s["value_heads"] * s["value_dim"]
    hv = s["value_heads"]
    conv_w = dev(_inputs.normal(90, 1, (width, conv), 0.5).astype(np.float16))
    a_log = dev(_inputs.normal(90, 2, (hv,), 0.5))
    dt_bias = dev(_inputs.normal(90, 3, (hv,), 0.5))
    q_norm = dev(_inputs.normal(90, 4, (s["head_dim"],), 0.1))
    k_norm = dev(_inputs.normal(90, 5, (s["head_dim"],), 0.1))

    session = ops.AttentionSession(PRODUCER_KINDS, batch, capacity, **SHAPE)
    session.set_producers(rotary_dim=rot, rope_theta=theta, conv_kernel=conv)
    # The composed reference: its own caches, state and conv history.
    keys = torch.zeros(batch, capacity, s["kv_heads"], s["head_dim"], dtype=torch.float16,
                       device="cuda")
    values = torch.zeros_like(keys)
    state = torch.zeros(batch, hv, s["key_dim"], s["value_dim"], device="cuda")
    hist = torch.zeros(batch, width, conv - 1, dtype=torch.float16, device="cuda")
    past = 0
    for step, tokens in enumerate([40, 1, 3]):
        delta, gqa = projection_inputs(batch, tokens, 91 + step)
        out_d = torch.full((batch, tokens, hv * s["value_dim"]), float("nan"),
                           dtype=torch.float16, device="cuda")
        out_g = torch.full((batch, tokens, s["query_heads"], s["head_dim"]), float("nan"),
                           dtype=torch.float16, device="cuda")
        layers = [ops.LayerProjections(out=out_d, conv_weight=conv_w, a_log=a_log,
                                       dt_bias=dt_bias, **delta),
                  ops.LayerProjections(out=out_g, q_norm=q_norm, k_norm=k_norm, **gqa)]
        session.step_projections(tokens, layers, trace_plan=True)
        torch.cuda.synchronize()

        q, k, v = ops.delta_prepare(delta["qkv"], conv_w, hist, s["key_heads"], s["key_dim"],
                                    hv, s["value_dim"])
        beta, decay = ops.delta_gates(delta["a"], delta["b"], a_log, dt_bias)
        ref_d = ops.delta_update(q, k, v, beta, decay, state)
        qr = ops.norm_rope(gqa["qg"], q_norm, past, rot, theta, head_dim=s["head_dim"])
        ops.norm_rope(gqa["k"], k_norm, past, rot, theta, out=keys, output_start=past)
        ops.cache_append(gqa["v"], values, past)
        ref_g = (ops.gqa_prefill(qr, keys, values, past) if tokens > 1
                 else ops.gqa_decode(qr, keys, values, past))
        torch.cuda.synchronize()
        past += tokens

        assert torch.equal(out_d, ref_d), step
        assert torch.equal(out_g, ref_g), step
        assert session.past == past
        assert torch.equal(session.read_state(0, abi.STATE_RECURRENT), state)
        assert torch.equal(session.read_state(0, abi.STATE_CONV_HISTORY), hist)
        assert torch.equal(session.read_state(1, abi.STATE_KEYS), keys)
        assert torch.equal(session.read_state(1, abi.STATE_VALUES), values)
        kernels = [d["kernel"] for d in session.plan()]
        assert kernels[:3] == ["deltaPrepare", "deltaGates", "graphDeltaUpdate"]
        assert kernels[3:6] == ["normRope", "normRope", "cacheAppend"]
        assert kernels[6:] == (["gqaFlashAttention"] if tokens > 1 else ["gqaScores", "gqaSoftmax"])

    session.reset()
    assert not session.read_state(0, abi.STATE_CONV_HISTORY).any()
    session.close()


def test_step_projections_needs_producer_settings():
    session = ops.AttentionSession(PRODUCER_KINDS, 1, 8, **SHAPE)
    delta, gqa = projection_inputs(1, 2, 7)
    out = torch.empty(1, 2, 512, dtype=torch.float16, device="cuda")
    layers = [ops.LayerProjections(out=out, **delta), ops.LayerProjections(out=out, **gqa)]
    with pytest.raises(abi.LlmiError) as err:
        session.step_projections(2, layers)
    assert err.value.status == abi.LLMI_INVALID_ARGUMENT
    assert session.past == 0 and not session.invalid
    session.close()


def test_set_producers_checks_its_settings():
    session = ops.AttentionSession(PRODUCER_KINDS, 1, 8, **SHAPE)
    with pytest.raises(abi.LlmiError) as err:
        session.set_producers(rotary_dim=63)          # odd rotary width
    assert err.value.status == abi.LLMI_UNSUPPORTED
    with pytest.raises(abi.LlmiError) as err:
        session.set_producers(conv_kernel=1)          # no conv history
    assert err.value.status == abi.LLMI_UNSUPPORTED
    session.set_producers()
    with pytest.raises(abi.LlmiError) as err:
        session.set_producers()                       # once per session
    assert err.value.status == abi.LLMI_INVALID_ARGUMENT
    assert not session.read_state(0, abi.STATE_CONV_HISTORY).any()
    session.close()
