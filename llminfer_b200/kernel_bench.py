"""Kernel microbenchmark for the attention path (the CUDA counterpart of the
reference's llmi-metal-bench, tools/metal-bench/Benchmark.h:12-47).

Times one op of the C ABI with CUDA events on its stream: warm-up, then the
best and median of N samples.  Inputs are seeded synthetic tensors on the
device; unless --no-check, a few rows are verified against a plain PyTorch
fp32 evaluation of the same op first (as metal-bench verifies sampled outputs
on the CPU before timing).  Prints one JSON object.

  python -m llminfer_b200.kernel_bench decode  --batch 64 --past 4096 --capacity 8192
  python -m llminfer_b200.kernel_bench prefill --batch 1 --tokens 128
  python -m llminfer_b200.kernel_bench delta   --batch 256 --tokens 1 --state-std 0.02
  python -m llminfer_b200.kernel_bench delta   --batch 4 --tokens 4096 [--no-scratch]
  python -m llminfer_b200.kernel_bench append  --batch 64 --tokens 1 --past 4096
  python -m llminfer_b200.kernel_bench rope    --batch 16 --tokens 8192 --past 0
  python -m llminfer_b200.kernel_bench deltaprep --batch 16 --tokens 8192
  python -m llminfer_b200.kernel_bench step --batch 2 --past 8320 --capacity 8448
  python -m llminfer_b200.kernel_bench traffic --csv launches.csv --workload decode \
      --batch 64 --past 4096 --capacity 8192 [--out profiles/traffic_c2_decode.jsonl]
"""
from __future__ import annotations

import argparse
import json
import math
import statistics
from pathlib import Path

import torch

from . import ops

ROOT = Path(__file__).resolve().parent.parent


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def time_fn(fn, samples: int, warmup: int):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(samples)]
    for a, b in events:
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    ms = sorted(a.elapsed_time(b) for a, b in events)
    return ms[0], statistics.median(ms)


def time_graph(fn, reps: int = 50):
    """Device time per call of fn captured once into a CUDA graph and replayed
    `reps` times back to back between two events (no Python wrapper per call):
    the measure for launch-bound shapes."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def torch_gqa(q, kc, vc, past, rows):
    """fp32 causal GQA for the listed (seq, token, head) rows."""
    B, T, Hq, D = q.shape
    g = Hq // kc.shape[2]
    out = []
    for s, t, h in rows:
        n = past + t + 1
        k = kc[s, :n, h // g].float()
        v = vc[s, :n, h // g].float()
        w = torch.softmax(k @ q[s, t, h].float() / math.sqrt(D), dim=0)
        out.append(w @ v)
    return torch.stack(out)


def errors(a, b):
    d = (a.double() - b.double())
    return float(d.abs().max()), float(d.norm() / b.double().norm().clamp_min(1e-300))


def bench_gqa(args, decode: bool):
    gen = torch.Generator(device="cuda").manual_seed(args.seed)
    B, T = args.batch, 1 if decode else args.tokens
    Hq, Hkv, D = args.heads[0], args.heads[1], args.dim
    cap = max(args.capacity, args.past + T)
    kc = torch.randn(B, cap, Hkv, D, generator=gen, device="cuda").half()
    vc = torch.randn(B, cap, Hkv, D, generator=gen, device="cuda").half()
    q = torch.randn(B, T, Hq, D, generator=gen, device="cuda").half()
    out = torch.empty_like(q)
    if decode:
        ws = torch.empty(ops.decode_workspace_bytes(B, Hq, Hkv, D, args.past), dtype=torch.uint8,
                         device="cuda")
        fn = lambda: ops.gqa_decode(q, kc, vc, args.past, out=out, workspace=ws)
    else:
        fn = lambda: ops.gqa_prefill(q, kc, vc, args.past, out=out)
    check = None
    if not args.no_check:
        fn()
        rows = [(s, t, h) for s in {0, B - 1} for t in {0, T - 1} for h in {0, Hq - 1}]
        want = torch_gqa(q, kc, vc, args.past, rows)
        got = torch.stack([out[s, t, h].float() for s, t, h in rows])
        check = dict(zip(("max_abs", "rel_l2"), errors(got, want)))
    best, med = time_fn(fn, args.samples, args.warmup)
    graph_ms = time_graph(fn) if args.graph else None
    rows_read = args.past + T
    nbytes = B * (2 * T * Hq * D * 2 + 2 * rows_read * Hkv * D * 2)
    pairs = T * args.past + T * (T + 1) // 2
    flops = 2 * 2 * B * Hq * pairs * D
    hbm, tf, src = peaks()
    res = dict(op="gqaScores+gqaSoftmax" if decode else "gqaFlashAttention", batch=B, tokens=T,
               past=args.past, heads=[Hq, Hkv], dim=D, best_ms=best, median_ms=med,
               gbs=nbytes / (med * 1e-3) / 1e9, tflops=flops / (med * 1e-3) / 1e12,
               hbm_frac=nbytes / (med * 1e-3) / 1e9 / hbm, tensor_frac=flops / (med * 1e-3) / 1e12 / tf,
               peaks=src, check=check)
    if graph_ms is not None:
        res.update(graph_ms=graph_ms, graph_gbs=nbytes / (graph_ms * 1e-3) / 1e9,
                   graph_hbm_frac=nbytes / (graph_ms * 1e-3) / 1e9 / hbm)
    return res


def bench_delta(args):
    gen = torch.Generator(device="cuda").manual_seed(args.seed)
    B, T = args.batch, args.tokens
    Hk, Hv, dk, dv = args.delta_heads[0], args.delta_heads[1], args.delta_dims[0], args.delta_dims[1]
    nrm = torch.nn.functional.normalize
    q = (nrm(torch.randn(B, T, Hk, dk, generator=gen, device="cuda"), dim=-1) / dk ** 0.5)
    q = q.reshape(B, T, Hk * dk).contiguous()
    k = nrm(torch.randn(B, T, Hk, dk, generator=gen, device="cuda"), dim=-1).reshape(B, T, Hk * dk).contiguous()
    v = torch.randn(B, T, Hv * dv, generator=gen, device="cuda").half()
    beta = torch.sigmoid(torch.randn(B, T, Hv, generator=gen, device="cuda")).half().float()
    decay = torch.exp(-torch.nn.functional.softplus(torch.randn(B, T, Hv, generator=gen, device="cuda")))
    state0 = torch.randn(B, Hv, dk, dv, generator=gen, device="cuda") * args.state_std
    state = state0.clone()
    out = torch.empty_like(v)
    if args.no_scratch:
        ws = False  # llmi_cuda_delta_update: one kernel per head, no scratch
    else:
        ws = torch.empty(max(16, ops.delta_workspace_bytes(B, T, Hk, dk, Hv, dv)),
                         dtype=torch.uint8, device="cuda")
    fn = lambda: ops.delta_update(q, k, v, beta, decay, state, out=out, workspace=ws)
    check = None
    if not args.no_check:
        fn()
        s = 0
        S = state0[s].double().clone()
        ys = []
        g = Hv // Hk
        for t in range(T):
            kt = k[s, t].double().reshape(Hk, dk).repeat_interleave(g, 0)
            qt = q[s, t].double().reshape(Hk, dk).repeat_interleave(g, 0)
            a = decay[s, t].double()[:, None, None]
            S = S * a
            pred = torch.einsum("hij,hi->hj", S, kt)
            delta = (v[s, t].double().reshape(Hv, dv) - pred) * beta[s, t].double()[:, None]
            S = S + kt[:, :, None] * delta[:, None, :]
            ys.append(torch.einsum("hij,hi->hj", S, qt).reshape(-1))
        e_out = errors(out[s].float(), torch.stack(ys).float())
        e_state = errors(state[s].float(), S.float())
        check = dict(out_max_abs=e_out[0], out_rel_l2=e_out[1], state_max_abs=e_state[0],
                     state_rel_l2=e_state[1])
    best, med = time_fn(fn, args.samples, args.warmup)
    nbytes = B * (2 * T * Hk * dk * 4 + T * Hv * dv * 2 + 2 * T * Hv * 4 + 2 * Hv * dk * dv * 4
                  + T * Hv * dv * 2)
    hbm, tf, src = peaks()
    return dict(op="graphDeltaUpdate", form="no scratch" if args.no_scratch else "scratch",
                batch=B, tokens=T, heads=[Hk, Hv], dims=[dk, dv],
                best_ms=best, median_ms=med, gbs=nbytes / (med * 1e-3) / 1e9,
                hbm_frac=nbytes / (med * 1e-3) / 1e9 / hbm,
                cost_model_tflops=2 * 3 * B * T * Hv * dk * dv / (med * 1e-3) / 1e12,
                peaks=src, check=check)


def bench_append(args):
    gen = torch.Generator(device="cuda").manual_seed(args.seed)
    B, T, Hkv, D = args.batch, args.tokens, args.heads[1], args.dim
    cap = max(args.capacity, args.past + T)
    cache = torch.zeros(B, cap, Hkv, D, dtype=torch.float16, device="cuda")
    rows = torch.randn(B, T, Hkv, D, generator=gen, device="cuda").half()
    fn = lambda: ops.cache_append(rows, cache, args.past)
    check = None
    if not args.no_check:
        fn()
        check = dict(exact=bool(torch.equal(cache[:, args.past:args.past + T], rows)))
    best, med = time_fn(fn, args.samples, args.warmup)
    nbytes = 2 * rows.numel() * 2
    return dict(op="cacheAppend", batch=B, tokens=T, best_ms=best, median_ms=med,
                gbs=nbytes / (med * 1e-3) / 1e9, check=check)


def bench_rope(args):
    """q and k of a GQA layer: normRope of q (sliced from [q | gate] rows) and
    of k (written into the key cache at row past)."""
    gen = torch.Generator(device="cuda").manual_seed(args.seed)
    B, T, (Hq, Hkv), D = args.batch, args.tokens, args.heads, args.dim
    rot = D // 4
    cap = max(args.capacity, args.past + T)
    qg = torch.randn(B, T, Hq, 2 * D, generator=gen, device="cuda").half()
    k = torch.randn(B, T, Hkv, D, generator=gen, device="cuda").half()
    wq = (0.1 * torch.randn(D, generator=gen, device="cuda")).float()
    wk = (0.1 * torch.randn(D, generator=gen, device="cuda")).float()
    qo = torch.empty(B, T, Hq, D, dtype=torch.float16, device="cuda")
    cache = torch.zeros(B, cap, Hkv, D, dtype=torch.float16, device="cuda")

    def fn():
        ops.norm_rope(qg, wq, args.past, rot, 1e7, head_dim=D, out=qo)
        ops.norm_rope(k, wk, args.past, rot, 1e7, out=cache, output_start=args.past)

    check = None
    if not args.no_check:
        fn()
        # fp32 RmsNorm (1 + w) and rotate-half RoPE, no intermediate rounding.
        x = qg[..., :D].float()
        x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * (1 + wq)
        pos = torch.arange(args.past, args.past + T, device="cuda").float()
        inv = 1.0 / (1e7 ** (torch.arange(0, rot, 2, device="cuda").float() / rot))
        ang = pos[:, None] * inv[None, :]
        c, s_ = ang.cos()[None, :, None, :], ang.sin()[None, :, None, :]
        x1, x2 = x[..., :rot // 2], x[..., rot // 2:rot]
        ref = torch.cat((x1 * c - x2 * s_, x2 * c + x1 * s_, x[..., rot:]), -1)
        m, r = errors(qo.float(), ref)
        check = dict(max_abs=m, rel_l2=r)
    best, med = time_fn(fn, args.samples, args.warmup)
    nbytes = (B * T * Hq * D * 2) * 2 + (B * T * Hkv * D * 2) * 2
    hbm, _, src = peaks()
    gbs = nbytes / (med * 1e-3) / 1e9
    return dict(op="normRope (q and k)", batch=B, tokens=T, heads=[Hq, Hkv], dim=D,
                rotary_dim=rot, best_ms=best, median_ms=med, gbs=gbs, hbm_frac=gbs / hbm,
                peaks=src, check=check)


def bench_deltaprep(args):
    """The DeltaNet block's q, k, v from its qkv projection (conv + SiLU +
    L2 norms) and its gates."""
    gen = torch.Generator(device="cuda").manual_seed(args.seed)
    B, T = args.batch, args.tokens
    (Hk, Hv), (dk, dv) = args.delta_heads, args.delta_dims
    W, K = 2 * Hk * dk + Hv * dv, 4
    qkv = torch.randn(B, T, W, generator=gen, device="cuda").half()
    wconv = (0.5 * torch.randn(W, K, generator=gen, device="cuda")).half()
    hist = torch.zeros(B, W, K - 1, dtype=torch.float16, device="cuda")
    a = torch.randn(B, T, Hv, generator=gen, device="cuda").half()
    b = torch.randn(B, T, Hv, generator=gen, device="cuda").half()
    a_log = torch.randn(Hv, generator=gen, device="cuda").float()
    dt_bias = torch.randn(Hv, generator=gen, device="cuda").float()

    def fn():
        ops.delta_prepare(qkv, wconv, hist, Hk, dk, Hv, dv)
        ops.delta_gates(a, b, a_log, dt_bias)

    check = None
    if not args.no_check:
        h0 = torch.zeros_like(hist)
        q, _, _ = ops.delta_prepare(qkv, wconv, h0, Hk, dk, Hv, dv)
        # fp32 depthwise conv + SiLU (no intermediate fp16 rounding), q L2 norm.
        x = torch.cat([torch.zeros_like(hist).float().transpose(1, 2), qkv.float()], 1)
        conv = sum(x[:, j:j + T] * wconv[:, j].float() for j in range(K))
        y = conv * torch.sigmoid(conv)
        qr = y[..., :Hk * dk].reshape(B, T, Hk, dk)
        qr = (qr * torch.rsqrt(qr.pow(2).sum(-1, keepdim=True) + 1e-6) / math.sqrt(dk))
        m, r = errors(q, qr.reshape(B, T, -1))
        check = dict(q_max_abs=m, q_rel_l2=r)
    best, med = time_fn(fn, args.samples, args.warmup)
    nbytes = B * T * (W * 2 + 2 * Hk * dk * 4 + Hv * dv * 2 + Hv * 2 * 2 + Hv * 2 * 4)
    hbm, _, src = peaks()
    gbs = nbytes / (med * 1e-3) / 1e9
    return dict(op="deltaPrepare + deltaGates", batch=B, tokens=T, heads=[Hk, Hv],
                dims=[dk, dv], best_ms=best, median_ms=med, gbs=gbs, hbm_frac=gbs / hbm,
                peaks=src, check=check)


# ---- measured DRAM traffic against the cost model (llmi graph --json counterpart) ----

# Kernel-name fragments of this library's launches -> (GraphIR op, --plan name).
# (ncu shows the names with or without their namespaces.)
KERNEL_DISPATCH = [
    ("cache_append", "KvAppend", "cacheAppend"),
    ("partial_", "CausalGqa", "gqaScores"),
    ("merge(", "CausalGqa", "gqaSoftmax"),
    ("gqa_prefill", "CausalGqa", "gqaFlashAttention"),
    ("solve_pass", "DeltaUpdate", "graphDeltaUpdate"),
    ("chunked_tc", "DeltaUpdate", "graphDeltaUpdate"),
    ("recurrent", "DeltaUpdate", "graphDeltaUpdate"),
]
# The launch that starts one call of each op (a call may launch several kernels).
CALL_MARKERS = {"KvAppend": "cache_append", "CausalGqa": ("partial_", "gqa_prefill"),
                "DeltaUpdate": ("chunked_tc", "recurrent")}


def read_ncu_csv(path):
    """Launches of an `ncu --csv` metrics file: [(id, kernel name, {metric: value})]."""
    import csv
    lines = [l for l in Path(path).read_text().splitlines() if l.startswith('"')]
    launches = {}
    for row in csv.DictReader(lines):
        key = row["ID"]
        name = row["Kernel Name"]
        value = float(row["Metric Value"].replace(",", ""))
        unit = row.get("Metric Unit", "")
        scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "nsecond": 1,
                 "usecond": 1e3, "msecond": 1e6}.get(unit, 1)
        launches.setdefault(key, (name, {}))[1][row["Metric Name"]] = value * scale
    return [(k, n, m) for k, (n, m) in launches.items()]


def traffic(args):
    """Per GraphIR op of one call: the DRAM bytes ncu measured for this library's
    kernels next to the cost model's logical bytes (llmi_cuda_describe_step, the
    reference's Cost.cpp:85-93), from an ncu CSV of gpu__time_duration.sum,
    dram__bytes_read.sum and dram__bytes_write.sum captured by hand."""
    from . import describe_step, make_stack_config
    launches = read_ncu_csv(args.csv)
    per_op = {}
    for _, name, metrics in launches:
        hit = next(((op, plan) for frag, op, plan in KERNEL_DISPATCH if frag in name), None)
        if hit is None:
            continue
        op, plan = hit
        entry = per_op.setdefault(op, {"calls": 0, "dispatches": {}})
        markers = CALL_MARKERS[op]
        markers = (markers,) if isinstance(markers, str) else markers
        if any(m in name for m in markers):
            entry["calls"] += 1
        d = entry["dispatches"].setdefault(plan, {"launches": 0, "time_ns": 0.0,
                                                  "dram_bytes": 0.0, "kernels": {}})
        t_ns = metrics.get("gpu__time_duration.sum", 0.0)
        nbytes = (metrics.get("dram__bytes_read.sum", 0.0)
                  + metrics.get("dram__bytes_write.sum", 0.0))
        d["launches"] += 1
        d["time_ns"] += t_ns
        d["dram_bytes"] += nbytes
        kern = d["kernels"].setdefault(name.split("(")[0].replace("void ", ""),
                                       {"launches": 0, "time_ns": 0.0, "dram_bytes": 0.0})
        kern["launches"] += 1
        kern["time_ns"] += t_ns
        kern["dram_bytes"] += nbytes
    # Logical bytes of one call of each op at the workload's shape.
    if args.workload == "delta":
        Hk, Hv = args.delta_heads
        dk, dv = args.delta_dims
        cfg, keep = make_stack_config([0], 1, args.tokens, key_heads=Hk, key_dim=dk,
                                      value_heads=Hv, value_dim=dv)
        step = json.loads(describe_step(cfg, args.tokens, 0))
    else:
        T = 1 if args.workload == "decode" else args.tokens
        cap = max(args.capacity, args.past + T)
        cfg, keep = make_stack_config([1], 1, cap, query_heads=args.heads[0],
                                      kv_heads=args.heads[1], head_dim=args.dim)
        step = json.loads(describe_step(cfg, T, args.past))
    logical = {op["kind"]: (op["cost"]["logical_read_bytes"] + op["cost"]["logical_write_bytes"])
               * args.batch for op in step["ops"]}
    lines = []
    for op, entry in per_op.items():
        calls = max(entry["calls"], 1)
        measured = sum(d["dram_bytes"] for d in entry["dispatches"].values()) / calls
        line = {"op": op, "workload": args.workload, "batch": args.batch, "calls": calls,
                "dispatches": {k: {"launches": v["launches"],
                                   "time_us_per_call": round(v["time_ns"] / calls / 1e3, 2),
                                   "dram_bytes_per_call": int(v["dram_bytes"] / calls),
                                   "kernels": {n: {"launches": kv["launches"],
                                                   "time_us_per_call":
                                                       round(kv["time_ns"] / calls / 1e3, 2),
                                                   "dram_bytes_per_call":
                                                       int(kv["dram_bytes"] / calls)}
                                               for n, kv in v["kernels"].items()}}
                               for k, v in entry["dispatches"].items()},
                "measured_dram_bytes_per_call": int(measured),
                "logical_bytes_per_call": logical.get(op),
                "measured_over_logical": (round(measured / logical[op], 4)
                                          if logical.get(op) else None)}
        lines.append(line)
    return lines


def bench_step(args):
    """One C5 decode step at `--batch` sequences, and its parts, each captured
    into a CUDA graph and replayed (device time per replay): 8 GQA layers (KvAppend
    + decode, through llmi_cuda_gqa_decode_append as the session issues them, and
    as three separate calls) and 24 recurrent DeltaNet layers, interleaved as in
    the hybrid stack (three DeltaNet layers, then one GQA layer).  The step
    is timed with and without LLMI_FLAG_SETTLED on its decode-path calls."""
    g = torch.Generator(device="cuda").manual_seed(args.seed)
    B, (Hq, Hkv), D, P, cap = args.batch, args.heads, args.dim, args.past, args.capacity
    (Hk, Hv), (dk, dv) = args.delta_heads, args.delta_dims
    layers, dlayers = args.layers, 3 * args.layers
    kc = [torch.randn(B, cap, Hkv, D, generator=g, device="cuda").half() for _ in range(layers)]
    vc = [torch.randn(B, cap, Hkv, D, generator=g, device="cuda").half() for _ in range(layers)]
    q = torch.randn(B, 1, Hq, D, generator=g, device="cuda").half()
    kn = torch.randn(B, 1, Hkv, D, generator=g, device="cuda").half()
    vn = torch.randn(B, 1, Hkv, D, generator=g, device="cuda").half()
    out = torch.empty_like(q)
    ws = torch.empty(ops.decode_workspace_bytes(B, Hq, Hkv, D, P), dtype=torch.uint8,
                     device="cuda")
    nrm = torch.nn.functional.normalize
    dq = nrm(torch.randn(B, 1, Hk, dk, generator=g, device="cuda"), dim=-1).reshape(B, 1, -1)
    dkk = nrm(torch.randn(B, 1, Hk, dk, generator=g, device="cuda"), dim=-1).reshape(B, 1, -1)
    dvv = torch.randn(B, 1, Hv * dv, generator=g, device="cuda").half()
    beta = torch.rand(B, 1, Hv, generator=g, device="cuda")
    decay = torch.rand(B, 1, Hv, generator=g, device="cuda") * 0.5 + 0.5
    states = [torch.randn(B, Hv, dk, dv, generator=g, device="cuda") * 0.02
              for _ in range(dlayers)]
    dout = torch.empty_like(dvv)

    dws = torch.empty(16, dtype=torch.uint8, device="cuda")  # T = 1 takes no scratch
    # Settled launches (LLMI_FLAG_SETTLED), as the session issues them: every
    # layer has its own caches and state, each appears once per captured
    # graph, and graph replays run one after another.
    settled = [True]

    def gqa(l, folded=True):
        if folded:
            ops.gqa_decode_append(q, kn, vn, kc[l], vc[l], P, out=out, workspace=ws,
                                  settled=settled[0])
        else:
            ops.cache_append(kn, kc[l], P)
            ops.cache_append(vn, vc[l], P)
            ops.gqa_decode(q, kc[l], vc[l], P, out=out, workspace=ws)

    def rec(l):
        ops.delta_update(dq, dkk, dvv, beta, decay, states[l], out=dout, workspace=dws,
                         settled=settled[0])

    def step(folded=True):
        for i in range(layers):
            for j in range(3):
                rec(3 * i + j)
            gqa(i, folded)

    def unsettled(fn):
        def run():
            settled[0] = False
            try:
                fn()
            finally:
                settled[0] = True
        return run

    reps = max(args.samples, 5)
    us = lambda fn, n=1: round(time_graph(fn, reps) * 1000 / n, 2)
    return {"op": "decode step", "batch": B, "heads": [Hq, Hkv], "dim": D, "past": P,
            "capacity": cap, "gqa_layers": layers, "delta_layers": dlayers,
            "delta_heads": [Hk, Hv], "delta_dims": [dk, dv],
            "us_step": us(step), "us_step_unsettled": us(unsettled(step)),
            "us_step_separate_appends": us(lambda: step(False)),
            "us_gqa_layer": us(lambda: [gqa(l) for l in range(layers)], layers),
            "us_gqa_layer_separate_appends":
                us(lambda: [gqa(l, False) for l in range(layers)], layers),
            "us_delta_layer": us(lambda: [rec(l) for l in range(dlayers)], dlayers),
            "timing": "each part captured into one CUDA graph, replayed back to back"}


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("op", choices=["decode", "prefill", "delta", "append", "rope", "deltaprep",
                                  "step", "traffic"])
    p.add_argument("--csv", help="traffic: ncu --csv file of gpu__time_duration.sum, "
                                 "dram__bytes_read.sum, dram__bytes_write.sum")
    p.add_argument("--workload", choices=["decode", "prefill", "delta"], default="decode",
                   help="traffic: the shape the CSV was captured at (same flags as the op)")
    p.add_argument("--out", help="traffic: also write the JSON lines to this file")
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--tokens", type=int, default=128)
    p.add_argument("--past", type=int, default=4096)
    p.add_argument("--capacity", type=int, default=8192)
    p.add_argument("--heads", type=int, nargs=2, default=[16, 4], metavar=("HQ", "HKV"))
    p.add_argument("--dim", type=int, default=256)
    p.add_argument("--delta-heads", type=int, nargs=2, default=[16, 32], metavar=("HK", "HV"))
    p.add_argument("--delta-dims", type=int, nargs=2, default=[128, 128], metavar=("DK", "DV"))
    p.add_argument("--state-std", type=float, default=0.0)
    p.add_argument("--samples", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--seed", type=int, default=179531)
    p.add_argument("--no-check", action="store_true")
    p.add_argument("--graph", action="store_true",
                   help="decode/prefill: also time the call replayed from a CUDA graph")
    p.add_argument("--layers", type=int, default=8,
                   help="step: GQA layers (three DeltaNet layers each)")
    p.add_argument("--no-scratch", action="store_true",
                   help="delta: the entry point without scratch (llmi_cuda_delta_update)")
    args = p.parse_args(argv)
    if args.op == "traffic":  # host only: no GPU needed
        lines = traffic(args)
        text = "\n".join(json.dumps(l) for l in lines) + "\n"
        if args.out:
            Path(args.out).write_text(text)
        print(text, end="")
        return
    torch.cuda.set_device(0)
    if args.op == "decode":
        res = bench_gqa(args, decode=True)
    elif args.op == "prefill":
        res = bench_gqa(args, decode=False)
    elif args.op == "delta":
        res = bench_delta(args)
    elif args.op == "rope":
        res = bench_rope(args)
    elif args.op == "deltaprep":
        res = bench_deltaprep(args)
    elif args.op == "step":
        res = bench_step(args)
    else:
        res = bench_append(args)
    ops.poll_error()
    print(json.dumps(res))


if __name__ == "__main__":
    main()
