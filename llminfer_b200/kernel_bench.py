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
  python -m llminfer_b200.kernel_bench append  --batch 64 --tokens 1 --past 4096
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
    fn = lambda: ops.delta_update(q, k, v, beta, decay, state, out=out)
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
    return dict(op="graphDeltaUpdate", batch=B, tokens=T, heads=[Hk, Hv], dims=[dk, dv],
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


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("op", choices=["decode", "prefill", "delta", "append"])
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
    args = p.parse_args(argv)
    torch.cuda.set_device(0)
    if args.op == "decode":
        res = bench_gqa(args, decode=True)
    elif args.op == "prefill":
        res = bench_gqa(args, decode=False)
    elif args.op == "delta":
        res = bench_delta(args)
    else:
        res = bench_append(args)
    ops.poll_error()
    print(json.dumps(res))


if __name__ == "__main__":
    main()
