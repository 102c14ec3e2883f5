"""The hybrid stack (llminfer_b200/stack.py) on one GPU: its layers against the
CPU oracle, and the (sequence x head) shards of 2 and 4 ranks - run one after
another on this GPU, reassembled with the all-gather layout - against the
unsharded run.
"""
import numpy as np
import pytest
import torch

import _inputs
import _oracle
from llminfer_b200 import stack as S

pytestmark = pytest.mark.gpu

# Hq * D == Hv * dv so every layer's head output has the same width.
SHAPE = dict(query_heads=4, kv_heads=2, head_dim=256, key_heads=4, key_dim=128,
             value_heads=8, value_dim=128)
KINDS = S.qwen35_kinds(4)  # three DeltaNet layers, then GQA
BATCH, PREFILL, DECODE = 4, 80, 3


def run_shard(world, rank, split="heads"):
    plan = S.ShardPlan.make(world, rank, BATCH, SHAPE, split)
    run = S.StackRun(torch, KINDS, BATCH, PREFILL, DECODE, SHAPE, plan, dist=None, seed=11)
    try:
        run.run_prefill()
        dec = []
        for s in range(DECODE):
            run.run_decode_step(s)
            run.join()
            torch.cuda.synchronize()
            dec.append(run.dec_out[s & 1].clone())
        run.session.sync()
        pre = [o.clone() for o in run.pre_out]
        operands = run.pre_in
        return plan, pre, torch.stack(dec), operands
    finally:
        run.close()


def host(t):
    return t.float().cpu().numpy() if t.dtype == torch.float16 else t.cpu().numpy()


def check(got, want):
    max_abs, rel = _inputs.errors(got, want)
    assert max_abs <= _inputs.MAX_ABS and rel <= _inputs.REL_L2, (max_abs, rel)


def test_stack_layers_match_oracle():
    plan, pre, dec, x = run_shard(1, 0)
    # DeltaNet layer 0: prefill from a zero state.
    d = {n: t.cpu().numpy() for n, t in x[0].items()}
    state0 = np.zeros((BATCH, SHAPE["value_heads"], 128, 128), np.float32)
    want, _ = _oracle.delta_update(d["q"], d["k"], d["v"], d["beta"], d["decay"], state0)
    check(host(pre[0]), want.reshape(BATCH, PREFILL, -1))
    # GQA layer 3: causal prefill over the rows it appended at past 0.
    g = {n: t.cpu().numpy() for n, t in x[3].items()}
    want = _oracle.gqa_dense(g["q"], g["k"], g["v"], 0)
    check(host(pre[3]), want.reshape(BATCH, PREFILL, -1))


@pytest.mark.parametrize("world,split", [(2, "heads"), (4, "heads"), (2, "sequences"),
                                         (4, "sequences")])
def test_sharded_stack_reassembles_to_unsharded(world, split):
    _, pre1, dec1, _ = run_shard(1, 0)
    shards = [run_shard(world, r, split) for r in range(world)]
    plan = shards[0][0]
    for layer in range(len(KINDS)):
        gathered = torch.stack([s[1][layer] for s in shards])
        full = S.unshard(gathered, world, plan.seq_groups, plan.head_groups)
        check(host(full), host(pre1[layer]))
    for step in range(DECODE):
        for layer in range(len(KINDS)):
            gathered = torch.stack([s[2][step][layer] for s in shards])
            full = S.unshard(gathered, world, plan.seq_groups, plan.head_groups)
            check(host(full), host(dec1[step][layer]))


def test_stack_benchmark_runs_and_reports():
    r = S.run_stack(torch, None, 1, 0, batch=2, prefill=96, decode=4, layers=8, shape=SHAPE)
    assert r["prefill_ms"] > 0 and r["decode_ms"] > 0
    assert r["cost_model"]["prefill_gflop"] > 0 and r["decode_tok_s"] > 0


def test_decode_steps_replayed_from_cuda_graphs_match_enqueue():
    plan = S.ShardPlan.make(1, 0, BATCH, SHAPE)
    run = S.StackRun(torch, KINDS, BATCH, PREFILL, DECODE, SHAPE, plan, dist=None, seed=13)
    try:
        def decode_outputs():
            run.run_prefill()
            outs = []
            for s in range(DECODE):
                run.run_decode_step(s)
                run.join()
                torch.cuda.synchronize()
                outs.append(run.dec_out[s & 1].clone())
            return torch.stack(outs)

        eager = decode_outputs()
        run.reset()
        run.run_prefill()
        run.capture_decode()
        run.reset()
        replayed = decode_outputs()
        run.session.sync()
        assert torch.equal(eager, replayed)
    finally:
        run.close()
