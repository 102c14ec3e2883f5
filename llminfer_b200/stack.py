"""Hybrid attention-stack benchmark on 1..N GPUs: the CUDA counterpart of
llmi-benchmark (tools/benchmark/Main.cpp:58-111) restricted to the attention
ops of the Qwen3.5-4B backbone: 24 Gated-DeltaNet layers and 8 GQA layers,
GQA at every fourth layer (the model's layer_types, docs/architecture.md:115).

As in llmi-benchmark, a session is opened with capacity = prefill + decode
tokens, warmed up with a short prefill and one decode step, reset, and then
one prefill step of `prefill` tokens and `decode` single-token steps are
timed.  The operands of every layer are seeded synthetic streams generated on
the device (GQA q/k/v ~ N(0,1) fp16; DeltaNet q, k = L2-normalised N(0,1)
with q scaled by 1/sqrt(dk), v ~ N(0,1) fp16, beta = half(sigmoid(N(0,1))),
decay = exp(-softplus(N(0,1)))); two operand sets per layer kind alternate
between layers, so consecutive layers never read the same buffers.

One process per GPU.  The (sequence x head) units are split as N = Ns x Nh.
The config's head sharding ("heads") takes Nh head groups (the largest
divisor of N that divides every head count) and Ns = N / Nh sequence groups;
the sequence-major split ("sequences") gives every rank whole sequences
(Nh = 1), so no collective is needed at all.  Rank r owns sequence group r // Nh and head
group r % Nh and opens an AttentionSession over that shard (B/Ns sequences,
H/Nh of every head count; head group g of the GQA layers holds query heads
[g Hq/Nh, (g+1) Hq/Nh) and their KV heads, of the DeltaNet layers value heads
[g Hv/Nh, ...) and their key heads, so the kernels' head-to-group mapping is
unchanged).  After each prefill layer the Nh ranks of a sequence group
all-gather that layer's head outputs over NCCL on a second stream, started
from the layer's completion event (llmi_cuda_session_set_layer_events) so it
overlaps the following layers; in decode the 32 layers' head outputs of a step
are gathered by one collective per step.  A gathered buffer is rank-major
[Nh][B/Ns][T][H/Nh * D] (of all N ranks, [N][...], when every rank's shard is
gathered); `unshard` turns it back into [B/Ns][T][H * D] ([B][T][H * D]).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import time
from dataclasses import dataclass

LAYER_DELTANET, LAYER_GQA = 0, 1
SEED = 179531

QWEN35_4B = dict(query_heads=16, kv_heads=4, head_dim=256, key_heads=16, key_dim=128,
                 value_heads=32, value_dim=128)


def qwen35_kinds(layers: int = 32, interval: int = 4) -> list[int]:
    """Layer kinds with full attention at every `interval`-th layer (3:1 for Qwen3.5)."""
    return [LAYER_GQA if (l + 1) % interval == 0 else LAYER_DELTANET for l in range(layers)]


@dataclass(frozen=True)
class ShardPlan:
    world: int
    rank: int
    seq_groups: int
    head_groups: int

    @classmethod
    def make(cls, world: int, rank: int, batch: int, shape: dict,
             split: str = "heads") -> "ShardPlan":
        """split "heads": as many head groups as divide every head count (the
        config's head sharding, with a collective per layer); "sequences":
        whole sequences per rank (Nh = 1), no collective."""
        if not 0 <= rank < world:
            raise ValueError(f"rank {rank} outside world {world}")
        if split == "sequences":
            if batch % world:
                raise ValueError(f"batch {batch} does not split over {world} ranks")
            return cls(world, rank, world, 1)
        if split != "heads":
            raise ValueError(f"unknown split {split!r}")
        g = 0
        for h in ("query_heads", "kv_heads", "key_heads", "value_heads"):
            g = math.gcd(g, shape[h])
        for nh in range(world, 0, -1):
            if world % nh == 0 and g % nh == 0 and batch % (world // nh) == 0:
                return cls(world, rank, world // nh, nh)
        raise ValueError(f"no (sequence x head) split of batch {batch} and heads {shape} "
                         f"over {world} ranks")

    @property
    def seq_group(self) -> int:
        return self.rank // self.head_groups

    @property
    def head_group(self) -> int:
        return self.rank % self.head_groups

    def seqs(self, batch: int) -> slice:
        n = batch // self.seq_groups
        return slice(self.seq_group * n, (self.seq_group + 1) * n)

    def heads(self, count: int) -> slice:
        n = count // self.head_groups
        return slice(self.head_group * n, (self.head_group + 1) * n)

    def shard_shape(self, shape: dict) -> dict:
        out = dict(shape)
        for h in ("query_heads", "kv_heads", "key_heads", "value_heads"):
            out[h] = shape[h] // self.head_groups
        return out


def head_group_ranks(plan: ShardPlan, seq_group: int) -> list:
    """The ranks holding the head shards of sequence group `seq_group`."""
    return [seq_group * plan.head_groups + h for h in range(plan.head_groups)]


def make_gather_group(dist, plan: ShardPlan):
    """The process group this rank's head outputs are all-gathered in: its
    sequence group's head shards (every rank takes part in creating each
    group, in the same order).  None: all ranks (one sequence group)."""
    if plan.seq_groups == 1:
        return None
    groups = [dist.new_group(head_group_ranks(plan, g)) for g in range(plan.seq_groups)]
    return groups[plan.seq_group]


def unshard(gathered, world: int, seq_groups: int, head_groups: int):
    """[N][B/Ns][T][H/Nh * D] (rank-major, as all-gathered) -> [B][T][H * D]."""
    _, b, t, w = gathered.shape
    x = gathered.reshape(seq_groups, head_groups, b, t, w)
    return x.permute(0, 2, 3, 1, 4).reshape(seq_groups * b, t, head_groups * w)


# ---------------------------------------------------------------------------
# operands


def _gen(torch, device, seed, tensor_id):
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1_000_003 + tensor_id) % (1 << 63))
    return g


def gqa_operands(torch, device, plan: ShardPlan, batch, tokens, shape, seed):
    """q [b, T, Hq/Nh, D], k/v [b, T, Hkv/Nh, D] fp16: the shard of full seeded tensors."""
    sq, D = plan.seqs(batch), shape["head_dim"]
    out = {}
    for tid, (name, heads) in enumerate((("q", "query_heads"), ("k", "kv_heads"),
                                         ("v", "kv_heads"))):
        full = torch.randn(batch, tokens, shape[heads], D, device=device,
                           generator=_gen(torch, device, seed, tid)).half()
        out[name] = full[sq, :, plan.heads(shape[heads])].contiguous()
        del full
    return out


def delta_operands(torch, device, plan: ShardPlan, batch, tokens, shape, seed):
    """q/k [b, T, Hk/Nh * dk] f32, v [b, T, Hv/Nh * dv] f16, beta/decay [b, T, Hv/Nh] f32."""
    F = torch.nn.functional
    sq = plan.seqs(batch)
    Hk, dk, Hv, dv = shape["key_heads"], shape["key_dim"], shape["value_heads"], shape["value_dim"]
    hk, hv = plan.heads(Hk), plan.heads(Hv)

    # Every transform runs on the full tensor before the shard is cut, so a
    # shard is bitwise the slice of the unsharded operands.
    def keys(tid, scale):
        full = torch.randn(batch, tokens, Hk, dk, device=device,
                           generator=_gen(torch, device, seed, tid))
        full = F.normalize(full, dim=-1, eps=1e-6) * scale
        x = full[sq, :, hk]
        return x.reshape(x.shape[0], tokens, -1).contiguous()

    def per_head(tid, fn):
        full = fn(torch.randn(batch, tokens, Hv, device=device,
                              generator=_gen(torch, device, seed, tid)))
        return full[sq, :, hv].contiguous()

    q = keys(10, dk ** -0.5)
    k = keys(11, 1.0)
    v = torch.randn(batch, tokens, Hv, dv, device=device,
                    generator=_gen(torch, device, seed, 12)).half()[sq, :, hv]
    v = v.reshape(v.shape[0], tokens, -1).contiguous()
    beta = per_head(13, lambda x: torch.sigmoid(x).half().float())
    decay = per_head(14, lambda x: torch.exp(-F.softplus(x)))
    return dict(q=q, k=k, v=v, beta=beta, decay=decay)


def layer_operands(torch, device, plan, kinds, batch, tokens, shape, seed, sets=2):
    """Per layer the operand dict; `sets` distinct sets per kind, alternating."""
    pool = {}
    for kind in (LAYER_GQA, LAYER_DELTANET):
        make = gqa_operands if kind == LAYER_GQA else delta_operands
        if kind in kinds:
            pool[kind] = [make(torch, device, plan, batch, tokens, shape,
                               seed * 10 + 2 * i + kind) for i in range(sets)]
    count = {LAYER_GQA: 0, LAYER_DELTANET: 0}
    layers = []
    for kind in kinds:
        layers.append(pool[kind][count[kind] % len(pool[kind])])
        count[kind] += 1
    return layers


def out_width(kind, shape):
    return (shape["query_heads"] * shape["head_dim"] if kind == LAYER_GQA
            else shape["value_heads"] * shape["value_dim"])


# ---------------------------------------------------------------------------
# runner


class StackRun:
    """One rank's shard of the stack: its session, operands, outputs and collectives."""

    def __init__(self, torch, kinds, batch, prefill, decode, shape, plan: ShardPlan,
                 dist=None, seed=SEED):
        from . import ops
        self.torch, self.ops, self.dist = torch, ops, dist
        self.kinds, self.batch, self.prefill, self.decode = list(kinds), batch, prefill, decode
        self.shape, self.plan = dict(shape), plan
        self.local = plan.shard_shape(shape)
        self.b = batch // plan.seq_groups
        self.device = torch.device("cuda", torch.cuda.current_device())
        widths = {out_width(k, self.local) for k in self.kinds}
        if len(widths) != 1:
            raise ValueError("GQA and DeltaNet head outputs must have the same width per token")
        self.width = widths.pop()
        self.session = ops.AttentionSession(self.kinds, self.b, prefill + decode, **self.local)
        self.stream = self.session.stream
        self.comm = torch.cuda.Stream(device=self.device)
        self.events = [torch.cuda.Event() for _ in self.kinds]
        for e in self.events:
            e.record(self.stream)
        self.session.set_layer_events(self.events)
        self.pre_in = layer_operands(torch, self.device, plan, self.kinds, batch, prefill, shape,
                                     seed)
        self.dec_in = layer_operands(torch, self.device, plan, self.kinds, batch, 1, shape,
                                     seed + 1)
        self.pre_out = [torch.empty(self.b, prefill, self.width, dtype=torch.float16,
                                    device=self.device) for _ in self.kinds]
        # Decode outputs of all layers of a step, double-buffered so step s+1
        # can run while step s is gathered.
        self.dec_out = [torch.empty(len(self.kinds), self.b, 1, self.width, dtype=torch.float16,
                                    device=self.device) for _ in range(2)]
        # The decode steps reuse the same buffers: build their operand tables once.
        self._dec_layers = [self._io(self.dec_in, [o[l] for l in range(len(self.kinds))])
                            for o in self.dec_out]
        self._dec_tables = [self.session.operand_table(x) for x in self._dec_layers]
        self.dec_free = [torch.cuda.Event() for _ in range(2)]
        for e in self.dec_free:
            e.record(self.comm)
        self.step_done = torch.cuda.Event()
        self.graphs = None  # per decode step, once capture_decode() has run
        n = plan.world
        # Without a process group (dist None) a multi-rank plan runs one
        # shard on this GPU and leaves the outputs unshared (emulation).  A
        # sequence-major split needs no collective: every rank holds all heads
        # of its sequences.
        self.gathering = dist is not None and n > 1 and plan.head_groups > 1
        self.pre_gathered = self.dec_gathered = None
        self.group = None
        if self.gathering:
            # Each sequence group gathers only its own head shards: a rank
            # receives (Nh - 1) / Nh of its sequences' outputs, nothing of the
            # other sequence groups'.
            self.group = make_gather_group(dist, plan)
            nh = plan.head_groups
            self.pre_gathered = torch.empty(nh, self.b, prefill, self.width,
                                            dtype=torch.float16, device=self.device)
            self.dec_gathered = torch.empty(nh, len(self.kinds), self.b, 1, self.width,
                                            dtype=torch.float16, device=self.device)

    def _io(self, operands, outs):
        ops = self.ops
        io = []
        for kind, x, out in zip(self.kinds, operands, outs):
            if kind == LAYER_GQA:
                o = out.view(self.b, -1, self.local["query_heads"], self.local["head_dim"])
                io.append(ops.LayerTensors(q=x["q"], k=x["k"], v=x["v"], out=o))
            else:
                io.append(ops.LayerTensors(q=x["q"], k=x["k"], v=x["v"], out=out,
                                           beta=x["beta"], decay=x["decay"]))
        return io

    def _gather(self, dst, src):
        torch = self.torch
        # The output is passed as the ranks' inputs concatenated along dim 0,
        # the form every backend accepts; dst itself is [N][...src.shape].
        with torch.cuda.stream(self.comm):
            self.dist.all_gather_into_tensor(dst.view(-1, *src.shape[1:]), src, group=self.group)

    def run_prefill(self, tokens=None, operands=None):
        """Enqueues one prefill step; per-layer gathers on the comm stream."""
        torch = self.torch
        tokens = self.prefill if tokens is None else tokens
        # Dense [b][tokens][width] views of the outputs (and of the gathered buffer).
        dense = lambda t, *lead: t.view(-1)[:math.prod(lead) * tokens * self.width].view(
            *lead, tokens, self.width)
        outs = [dense(o, self.b) for o in self.pre_out]
        if operands is None:
            operands = self.pre_in
        self.session._sync_inputs()
        self.session.enqueue(tokens, self._io(operands, outs))
        if self.gathering:
            for l, ev in enumerate(self.events):
                self.comm.wait_event(ev)
                self._gather(dense(self.pre_gathered, self.plan.head_groups, self.b), outs[l])
            self.stream.wait_stream(self.comm)

    def run_decode_step(self, step: int):
        torch = self.torch
        buf = step & 1
        out = self.dec_out[buf]
        if self.graphs is not None:
            # The step's launches and its all-gather are one graph.
            with torch.cuda.stream(self.stream):
                self.graphs[step].replay()
            return
        self.stream.wait_event(self.dec_free[buf])
        self.session.enqueue(1, self._dec_tables[buf])
        if self.gathering:
            self.step_done.record(self.stream)
            self.comm.wait_event(self.step_done)
            self._gather(self.dec_gathered, out)
        self.dec_free[buf].record(self.comm)

    def capture_decode(self):
        """Captures each decode step into its own CUDA graph (the step's `past`
        is part of its kernel arguments): the session's launches and, when the
        heads are sharded, the NCCL all-gather of the step's head outputs on
        the comm stream, joined back before the graph ends.  A step then costs
        the host one graph launch, with no per-step collective call from
        Python.  Every rank captures the same collectives in the same order.
        Call right after a prefill (the communicator exists by then):
        capturing runs nothing on the GPU but advances the session's `past`
        through every decode step, so reset the session and run the prefill
        again before replaying with run_decode_step."""
        torch = self.torch
        if self.session.past != self.prefill:
            raise RuntimeError("capture_decode needs the session right after a prefill")
        torch.cuda.synchronize()
        self.session.set_layer_events(None)
        graphs = []
        try:
            for step in range(self.decode):
                g = torch.cuda.CUDAGraph()
                buf = step & 1
                with torch.cuda.graph(g, stream=self.stream):
                    self.session.enqueue(1, self._dec_tables[buf])
                    if self.gathering:
                        self.step_done.record(self.stream)
                        self.comm.wait_event(self.step_done)
                        self._gather(self.dec_gathered, self.dec_out[buf])
                        self.stream.wait_stream(self.comm)
                graphs.append(g)
        finally:
            self.session.set_layer_events(self.events)
        self.graphs = graphs

    def join(self):
        self.stream.wait_stream(self.comm)

    def warmup(self):
        """llmi-benchmark's warm-up (a short prefill and one decode step), then reset."""
        short = [{n: t[:, :min(64, self.prefill)].contiguous() for n, t in x.items()}
                 for x in self.pre_in]
        self.run_prefill(tokens=min(64, self.prefill), operands=short)
        self.run_decode_step(0)
        self.join()
        self.session.sync()
        self.reset()

    def reset(self):
        self.torch.cuda.synchronize()
        self.session.reset()

    def gathered_prefill_output(self, layer):
        """[B / Ns][T][H*D]: every head of `layer`'s output for this rank's
        sequences, after a prefill (for checks)."""
        self.torch.cuda.synchronize()
        if not self.gathering:
            return self.pre_out[layer].clone()
        self._gather(self.pre_gathered, self.pre_out[layer])
        self.torch.cuda.synchronize()
        nh = self.plan.head_groups
        return unshard(self.pre_gathered, nh, 1, nh)

    def close(self):
        self.torch.cuda.synchronize()
        self.graphs = None
        self.session.set_layer_events(None)
        self.session.close()


def stack_costs(kinds, batch, prefill, decode, shape):
    """Reference cost model (Cost.cpp) of the prefill step and of all decode steps."""
    from . import describe_step, make_stack_config
    cfg, keep = make_stack_config(kinds, 1, prefill + decode, **shape)

    def one(tokens, past):
        d = json.loads(describe_step(cfg, tokens, past))
        macs = sum(op["cost"]["fp_macs"] for op in d["ops"]) * batch
        nbytes = sum(op["cost"]["logical_read_bytes"] + op["cost"]["logical_write_bytes"]
                     for op in d["ops"]) * batch
        gqa_macs = sum(op["cost"]["fp_macs"] for op in d["ops"]
                       if op["kind"] == "CausalGqa") * batch
        return macs, nbytes, gqa_macs

    pre = one(prefill, 0)
    dec_macs = dec_bytes = 0
    for s in range(decode):
        m, b, _ = one(1, prefill + s)
        dec_macs += m
        dec_bytes += b
    return dict(prefill_macs=pre[0], prefill_bytes=pre[1], prefill_gqa_macs=pre[2],
                decode_macs=dec_macs, decode_bytes=dec_bytes)


def run_stack(torch, dist, world, rank, batch=16, prefill=8192, decode=256, layers=32,
              shape=None, repeats=1, seed=SEED, graphs=True, split="heads"):
    """Times `repeats` (prefill, decode) runs; returns rank-0 metrics (max over ranks).
    With `graphs` the decode steps are replayed from CUDA graphs captured
    before the timed runs.  `split` picks the ShardPlan."""
    shape = dict(QWEN35_4B if shape is None else shape)
    kinds = qwen35_kinds(layers)
    plan = ShardPlan.make(world, rank, batch, shape, split)
    run = StackRun(torch, kinds, batch, prefill, decode, shape, plan, dist=dist, seed=seed)
    try:
        run.warmup()
        if graphs and decode > 0:
            run.run_prefill()
            run.capture_decode()
            run.reset()
        pre_ms, dec_ms, issue_ms = [], [], []
        for _ in range(repeats):
            if dist is not None and world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            ev[0].record(run.stream)
            run.run_prefill()
            ev[1].record(run.stream)
            # The decode steps are issued once the prefill has finished, so the
            # host time below is the issue cost alone (not time spent blocked
            # on a launch queue that the prefill keeps full).  The device
            # interval starts at ev[1], so it includes any host lag.
            run.join()
            run.stream.synchronize()
            t0 = time.perf_counter()
            for s in range(decode):
                run.run_decode_step(s)
            run.join()
            ev[2].record(run.stream)
            issue_ms.append((time.perf_counter() - t0) * 1e3)
            run.session.sync()
            torch.cuda.synchronize()
            p, d = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
            if dist is not None and world > 1:
                t = torch.tensor([p, d], dtype=torch.float64, device=run.device)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                p, d = float(t[0]), float(t[1])
            pre_ms.append(p)
            dec_ms.append(d)
            run.reset()
    finally:
        run.close()
    costs = stack_costs(kinds, batch, prefill, decode, shape)
    p, d = statistics.median(pre_ms), statistics.median(dec_ms)
    return {
        "workload": (f"C5 hybrid stack: {kinds.count(LAYER_DELTANET)} DeltaNet + "
                     f"{kinds.count(LAYER_GQA)} GQA layers, batch {batch}, prefill {prefill}, "
                     f"{decode} decode steps"),
        "sharding": {"split": split, "sequence_groups": plan.seq_groups,
                     "head_groups": plan.head_groups,
                     "collective": f"NCCL all-gather of head outputs among the "
                                   f"{plan.head_groups} ranks of each sequence group "
                                   "(prefill: per layer, overlapped; decode: all layers of a "
                                   "step in one, inside the step's CUDA graph)"
                     if world > 1 and plan.head_groups > 1 else
                     "none (whole sequences per GPU)" if world > 1 else "none (1 GPU)"},
        "prefill_ms": round(p, 3),
        "prefill_tok_s": round(batch * prefill / (p / 1e3), 1),
        "prefill_tflops": round(2 * costs["prefill_macs"] / (p / 1e3) / 1e12, 2),
        "decode_ms": round(d, 3),
        "decode_tok_s": round(batch * decode / (d / 1e3), 1),
        "decode_gbs": round(costs["decode_bytes"] / (d / 1e3) / 1e9, 1),
        # Host time to issue the decode steps after the prefill (rank 0): at or
        # above decode_ms means the device waited for the host.
        "decode_host_issue_ms": round(statistics.median(issue_ms), 3),
        "repeats": repeats,
        "decode_steps_from": ("CUDA graphs captured per step (launches and collective)"
                              if graphs else "session enqueue"),
        "cost_model": {"prefill_gflop": round(2 * costs["prefill_macs"] / 1e9, 1),
                       "prefill_gqa_gflop": round(2 * costs["prefill_gqa_macs"] / 1e9, 1),
                       "decode_gb": round(costs["decode_bytes"] / 1e9, 2)},
    }


def main():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--batch", type=int, default=16)
    p.add_argument("--prefill-tokens", type=int, default=8192)
    p.add_argument("--decode-tokens", type=int, default=256)
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--repeats", type=int, default=1)
    p.add_argument("--split", choices=["heads", "sequences"], default="heads")
    args = p.parse_args()
    import datetime

    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    try:
        r = run_stack(torch, dist, world, rank, args.batch, args.prefill_tokens,
                      args.decode_tokens, args.layers, repeats=args.repeats, split=args.split)
        if rank == 0:
            # llmi-benchmark's report lines (tools/benchmark/Main.cpp:50-56).
            for phase, tokens, ms in (("Prefill", args.prefill_tokens, r["prefill_ms"]),
                                      ("Decode", args.decode_tokens, r["decode_ms"])):
                print(f"{phase}: {tokens} tokens in {ms / 1e3:.6f} s, "
                      f"{args.batch * tokens / (ms / 1e3):.2f} tok/s (batch {args.batch}, "
                      f"{world} GPU{'s' if world > 1 else ''})")
            print(json.dumps(r), flush=True)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
