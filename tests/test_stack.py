"""Host logic of the multi-GPU hybrid stack (llminfer_b200/stack.py) on the CPU:
the (sequence x head) split, the rank-major gather layout and its inverse,
sharded operand generation, and a world-size-2 gloo all-gather of head
outputs reassembled into the full layer output.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from llminfer_b200 import stack as S

SMALL = dict(query_heads=4, kv_heads=2, head_dim=256, key_heads=4, key_dim=128,
             value_heads=8, value_dim=128)


def test_qwen35_layer_pattern():
    kinds = S.qwen35_kinds()
    assert len(kinds) == 32
    assert kinds.count(S.LAYER_GQA) == 8 and kinds.count(S.LAYER_DELTANET) == 24
    assert [l for l, k in enumerate(kinds) if k == S.LAYER_GQA] == list(range(3, 32, 4))


@pytest.mark.parametrize("world,seq_groups,head_groups", [(1, 1, 1), (2, 1, 2), (4, 1, 4),
                                                         (8, 2, 4)])
def test_shard_plan_qwen35(world, seq_groups, head_groups):
    plans = [S.ShardPlan.make(world, r, 16, S.QWEN35_4B) for r in range(world)]
    assert {(p.seq_groups, p.head_groups) for p in plans} == {(seq_groups, head_groups)}
    # Every (sequence, KV head) and (sequence, value head) unit is owned exactly once.
    for heads in ("kv_heads", "value_heads", "query_heads", "key_heads"):
        owned = set()
        for p in plans:
            for b in range(16)[p.seqs(16)]:
                for h in range(S.QWEN35_4B[heads])[p.heads(S.QWEN35_4B[heads])]:
                    assert (b, h) not in owned
                    owned.add((b, h))
        assert len(owned) == 16 * S.QWEN35_4B[heads]
    # Head groups keep the GQA / DeltaNet head-to-group mapping inside a shard.
    for p in plans:
        q, kv = p.heads(16), p.heads(4)
        assert q.start // 4 == kv.start and (q.stop - 1) // 4 == kv.stop - 1
        vh, kh = p.heads(32), p.heads(16)
        assert vh.start // 2 == kh.start and (vh.stop - 1) // 2 == kh.stop - 1


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sequence_major_plan(world):
    plans = [S.ShardPlan.make(world, r, 16, S.QWEN35_4B, "sequences") for r in range(world)]
    assert {(p.seq_groups, p.head_groups) for p in plans} == {(world, 1)}
    owned = [b for p in plans for b in range(16)[p.seqs(16)]]
    assert sorted(owned) == list(range(16))
    assert all(p.heads(32) == slice(0, 32) for p in plans)
    full = torch.randn(16, 3, 8, 4)
    gathered = torch.stack([full[p.seqs(16)].reshape(16 // world, 3, -1) for p in plans])
    assert torch.equal(S.unshard(gathered, world, world, 1), full.reshape(16, 3, -1))


def test_shard_plan_rejects_impossible_split():
    with pytest.raises(ValueError):
        S.ShardPlan.make(3, 0, 16, S.QWEN35_4B, "sequences")
    with pytest.raises(ValueError):
        S.ShardPlan.make(2, 0, 16, S.QWEN35_4B, "rows")
    with pytest.raises(ValueError):
        S.ShardPlan.make(3, 0, 16, S.QWEN35_4B)
    with pytest.raises(ValueError):
        S.ShardPlan.make(2, 2, 16, S.QWEN35_4B)


def _shards(full, world, batch):
    plans = [S.ShardPlan.make(world, r, batch, SMALL) for r in range(world)]
    b, t, h, d = full.shape
    return plans, torch.stack([full[p.seqs(b), :, p.heads(h)].reshape(b // p.seq_groups, t, -1)
                               for p in plans])


@pytest.mark.parametrize("world", [1, 2, 4])
def test_unshard_inverts_the_split(world):
    full = torch.randn(4, 5, 8, 16)
    plans, gathered = _shards(full, world, 4)
    back = S.unshard(gathered, world, plans[0].seq_groups, plans[0].head_groups)
    assert torch.equal(back, full.reshape(4, 5, -1))


@pytest.mark.parametrize("world,rank", [(2, 1), (4, 3)])
def test_sharded_operands_are_slices_of_the_full_ones(world, rank):
    cpu = torch.device("cpu")
    full = S.ShardPlan.make(1, 0, 4, SMALL)
    part = S.ShardPlan.make(world, rank, 4, SMALL)
    g1 = S.gqa_operands(torch, cpu, full, 4, 6, SMALL, seed=5)
    gp = S.gqa_operands(torch, cpu, part, 4, 6, SMALL, seed=5)
    assert torch.equal(gp["q"], g1["q"][part.seqs(4), :, part.heads(4)])
    assert torch.equal(gp["k"], g1["k"][part.seqs(4), :, part.heads(2)])
    d1 = S.delta_operands(torch, cpu, full, 4, 6, SMALL, seed=6)
    dp = S.delta_operands(torch, cpu, part, 4, 6, SMALL, seed=6)
    hk, hv, sq = part.heads(4), part.heads(8), part.seqs(4)
    assert torch.equal(dp["k"], d1["k"].view(4, 6, 4, 128)[sq, :, hk].reshape(dp["k"].shape))
    assert torch.equal(dp["v"], d1["v"].view(4, 6, 8, 128)[sq, :, hv].reshape(dp["v"].shape))
    assert torch.equal(dp["decay"], d1["decay"][sq, :, hv])
    # Operand conventions of the DeltaUpdate contract.
    assert d1["q"].dtype == torch.float32 and d1["v"].dtype == torch.float16
    norms = d1["k"].view(4, 6, 4, 128).norm(dim=-1)
    assert torch.allclose(norms, torch.ones_like(norms), atol=1e-5)
    assert torch.allclose(d1["q"].view(4, 6, 4, 128).norm(dim=-1), norms / 128 ** 0.5, atol=1e-6)
    assert ((d1["decay"] > 0) & (d1["decay"] < 1)).all()
    assert torch.equal(d1["beta"], d1["beta"].half().float())


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, full, result):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = S.ShardPlan.make(world, rank, full.shape[0], SMALL)
        b, t, h, d = full.shape
        mine = full[plan.seqs(b), :, plan.heads(h)].reshape(b // plan.seq_groups, t, -1)
        gathered = torch.empty(world, *mine.shape, dtype=mine.dtype)
        dist.all_gather_into_tensor(gathered.view(-1, *mine.shape[1:]), mine.contiguous())
        back = S.unshard(gathered, world, plan.seq_groups, plan.head_groups)
        result[rank] = bool(torch.equal(back, full.reshape(b, t, -1)))
    finally:
        dist.destroy_process_group()


def test_gloo_all_gather_reassembles_layer_output():
    world = 2
    full = torch.randn(4, 3, 8, 16)
    result = mp.Manager().dict()
    mp.spawn(_gather_worker, args=(world, _free_port(), full, result), nprocs=world, join=True)
    assert dict(result) == {0: True, 1: True}


def _group_gather_worker(rank, world, port, full, result):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = S.ShardPlan.make(world, rank, full.shape[0], SMALL)
        group = S.make_gather_group(dist, plan)
        b, t, h, d = full.shape
        mine = full[plan.seqs(b), :, plan.heads(h)].reshape(b // plan.seq_groups, t, -1)
        nh = plan.head_groups
        gathered = torch.empty(nh, *mine.shape, dtype=mine.dtype)
        dist.all_gather_into_tensor(gathered.view(-1, *mine.shape[1:]), mine.contiguous(),
                                    group=group)
        back = S.unshard(gathered, nh, 1, nh)
        want = full[plan.seqs(b)].reshape(b // plan.seq_groups, t, -1)
        result[rank] = (plan.seq_groups, nh, S.head_group_ranks(plan, plan.seq_group),
                        bool(torch.equal(back, want)))
    finally:
        dist.destroy_process_group()


def test_gloo_gather_within_each_sequence_group():
    """World 4 as 2 sequence groups x 2 head groups: each sequence group
    gathers its own head shards (ranks {0, 1} and {2, 3}) and reassembles all
    heads of its sequences."""
    world = 4
    full = torch.randn(4, 3, 8, 16)
    result = mp.Manager().dict()
    mp.spawn(_group_gather_worker, args=(world, _free_port(), full, result), nprocs=world,
             join=True)
    assert dict(result) == {0: (2, 2, [0, 1], True), 1: (2, 2, [0, 1], True),
                            2: (2, 2, [2, 3], True), 3: (2, 2, [2, 3], True)}


def _rank_loss_worker(rank, world, port, result):
    import datetime
    import time

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        os._exit(3)  # this rank is lost between steps: no collective of its own in flight
    plan = S.ShardPlan.make(world, rank, 4, SMALL)
    mine = torch.ones(4 // plan.seq_groups, 2, 16)
    gathered = torch.empty(world, *mine.shape)
    t0 = time.monotonic()
    try:
        dist.all_gather_into_tensor(gathered.view(-1, *mine.shape[1:]), mine)
        result[rank] = ("completed", time.monotonic() - t0)
    except Exception as exc:  # the survivor must see an error, not wait forever
        result[rank] = ("error: " + type(exc).__name__, time.monotonic() - t0)
    os._exit(0)


def test_lost_rank_surfaces_as_an_error_not_a_hang():
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_loss_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung on the collective of a lost peer"
    assert procs[1].exitcode == 3
    outcome, seconds = result[0]
    assert outcome.startswith("error"), outcome
    assert seconds < 60
