#!/usr/bin/env python
"""Benchmark of the B200 attention backend (one JSON line on rank 0).

Headline workload ("C2"): one GQA decode step per
sequence - cacheAppend of the new key/value rows, then split-K decode
attention (gqaScores + gqaSoftmax) over past 4096 cached tokens, with the
appends folded into the decode's two kernels as the session lowers them - for a batch
of 64 sequences per GPU, Hq 16 / Hkv 4 / head_dim 256, fp16 caches of
capacity 8192.  The metric is HBM throughput: the logical bytes of the
step's ops under the reference cost model (lib/GraphIR/Cost.cpp:85-93) per
second.  Multi-GPU runs shard sequences (weak scaling, no collective).

Keys of the line beyond the base contract:
  roofline      the decode op (gqaScores + gqaSoftmax launches), timed with
                CUDA events on its stream, against the measured HBM copy
                bandwidth of MEASURED_PEAKS.json
  cpu_baseline  the reference's scalar check code restated in oracle/ (dense
                fp64 causal GQA, cacheAppend), built -O3 -march=native on this
                host: the whole C2 step on every core, and 2 sequences on one
                thread (one_thread_value); every secondary C1-C4 line carries
                the same pair for its op
  e2e           the same step through the C-ABI calls with pinned host
                buffers: H2D of q and the new rows, D2H of the output, timed;
                the copies run on their own streams, double-buffered, under
                the neighbouring steps' kernels
  secondary     the other kernels of the path: C1 prefill (replicas), the
                prefill at the C5 layer shape and the producers of its operands
                (each whole on every GPU); C2, C3 and C4 as fixed jobs split
                over the N GPUs (strong scaling: 64 sequences, 128 (sequence,
                value head) units, 256 sequences), each with its time on one
                GPU and the efficiency against it
  stack         the C5 hybrid stack (llminfer_b200/stack.py): 24 DeltaNet +
                8 GQA layers, batch 16, prefill 8192 then 256 decode steps,
                split by (sequence x head) over the N GPUs with an NCCL
                all-gather of head outputs (strong scaling)
  stack_sequence_major  (N > 1) the same stack with whole sequences per GPU,
                which needs no collective
`--impl reference` runs the reference arm: the CPU restatement of the
reference's code (oracle/, "port") on the host cores, same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "GQA/DeltaNet attn TFLOP/s (prefill), HBM GB/s (decode) vs roofline, 1-8 GPU"
C2 = dict(batch=64, past=4096, capacity=8192, query_heads=16, kv_heads=4, head_dim=256)
# C5: the hybrid stack (24 DeltaNet + 8 GQA layers), a fixed job split over the GPUs.
C5 = dict(batch=16, prefill=8192, decode=256, layers=32)
FALLBACK_PEAKS = dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0)
SEED = 179531


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-secondary", action="store_true", help="skip C1/C3/C4 measurements")
    p.add_argument("--no-stack", action="store_true", help="skip the C5 hybrid-stack run")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    return p.parse_args()


# ---------------------------------------------------------------------------
# helpers


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return dict(hbm_gbs=float(data["hbm_gbs"]), bf16_tflops=float(data["bf16_tflops"]),
                    bf16_tflops_sustained=float(data.get("bf16_tflops_sustained",
                                                         data["bf16_tflops"])),
                    source="measured")
    return dict(FALLBACK_PEAKS, source="fallback")


def profile_traffic(name: str, op: str):
    """DRAM bytes per call of `op` from profiles/traffic_<name>.jsonl, the output of
    `kernel_bench traffic` over an ncu capture of the same workload (or None)."""
    path = ROOT / "profiles" / f"traffic_{name}.jsonl"
    if not path.exists():
        return None
    for text in path.read_text().splitlines():
        line = json.loads(text)
        if line.get("op") == op:
            return line["measured_dram_bytes_per_call"]
    return None


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled every 10 ms during the timed
    region and once more as it ends, read through NVML (read-only queries)."""

    REASONS = {  # NVML clocks-event reason bits
        0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
        0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown",
    }

    def __init__(self, torch, device):
        import threading
        self.samples = []
        self.max_mhz = None
        self.error = None
        self.stop = threading.Event()
        self.thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            want = str(torch.cuda.get_device_properties(device).uuid).lower()
            self.handle = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                uuid = pynvml.nvmlDeviceGetUUID(h)
                uuid = uuid.decode() if isinstance(uuid, bytes) else uuid
                if want and want in uuid.lower():
                    self.handle = h
            if self.handle is None:
                raise RuntimeError(f"no NVML device with uuid {want}")
            self.nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.thread = threading.Thread(target=self._run, daemon=True)
        except Exception as exc:  # NVML missing or no match: report, do not fail the bench
            self.error = f"clock sampling unavailable: {exc}"

    def _reasons(self):
        n = self.nvml
        for name in ("nvmlDeviceGetCurrentClocksEventReasons",
                     "nvmlDeviceGetCurrentClocksThrottleReasons"):
            if hasattr(n, name):
                return getattr(n, name)(self.handle)
        return 0

    def _sample(self):
        try:
            sm = self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM)
            self.samples.append((sm, self._reasons()))
            return True
        except Exception as exc:
            self.error = str(exc)
            return False

    def _run(self):
        while not self.stop.is_set():
            if not self._sample():
                return
            self.stop.wait(0.01)

    def __enter__(self):
        if self.thread is not None:
            self.thread.start()
        return self

    def __exit__(self, *exc):
        self.stop.set()
        if self.thread is not None:
            self.thread.join(timeout=2)
            self._sample()  # the end of the region

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz,
                    "reasons": [self.error or "no samples"]}
        reasons = sorted({name for _, bits in self.samples
                          for bit, name in self.REASONS.items() if bits & bit})
        return {"sm_mhz": statistics.median(s for s, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.samples)}


class Dist:
    def __init__(self, gpus: int):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist

    def barrier(self):
        if self.pg is not None:
            self.pg.barrier()

    def max(self, value: float) -> float:
        if self.pg is None:
            return value
        import torch
        t = torch.tensor([value], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


def step_bytes(cfg_kinds, tokens, past, capacity, batch, **shape):
    """Logical bytes and MACs of one step of the given layers (reference cost model)."""
    import llminfer_b200 as L
    cfg, keep = L.make_stack_config(cfg_kinds, 1, capacity, **shape)
    d = json.loads(L.describe_step(cfg, tokens, past))
    per_op = {}
    for op in d["ops"]:
        c = op["cost"]
        per_op.setdefault(op["kind"], [0, 0, 0])
        per_op[op["kind"]][0] += (c["logical_read_bytes"] + c["logical_write_bytes"]) * batch
        per_op[op["kind"]][1] += c["fp_macs"] * batch
    return per_op


# ---------------------------------------------------------------------------
# CPU baselines: the oracle port (oracle/oracle.c), the reference's scalar
# check code restated in C.  Nothing here loads llminfer_b200: the bytes and
# MACs are priced by the oracle's own restatement of the reference cost model.


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def native_oracle():
    """The oracle built -O3 -march=native on this host (portable build as a fallback),
    with OpenMP set to every core this process may use (a launcher such as torchrun
    sets OMP_NUM_THREADS=1 for its workers)."""
    import importlib
    cores = host_cores()
    os.environ["OMP_NUM_THREADS"] = str(cores)
    sys.path.insert(0, str(ROOT / "tests"))
    oracle = importlib.import_module("_oracle")
    out = Path(tempfile.gettempdir()) / f"llmi_oracle_native_{os.getpid()}.so"
    try:
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "native",
                        f"NATIVE_OUT={out}"], check=True, capture_output=True)
        lib = oracle.load(out)
        flags = "-O3 -march=native"
    except (subprocess.CalledProcessError, OSError):
        lib = oracle.load()
        flags = "-O3"
    lib.oracle_set_threads(cores)
    oracle._lib = lib
    return oracle, flags, cores


def c2_step_bytes(oracle, sequences: int) -> int:
    """Logical bytes of `sequences` sequences of the C2 step (KvAppend + CausalGqa)."""
    P, Hq, Hkv, D = C2["past"], C2["query_heads"], C2["kv_heads"], C2["head_dim"]
    kv = sum(oracle.kv_append_bytes(1, Hkv, D))
    gqa = sum(oracle.gqa_bytes(1, P, Hq, Hkv, D))
    return (kv + gqa) * sequences


def c2_host_inputs(sequences: int):
    """One seeded sequence of the C2 step repeated `sequences` times (the work does not
    depend on the values): q [n,1,Hq,D], new rows [n,1,Hkv,D], caches [n,P+1,Hkv,D]."""
    import numpy as np
    sys.path.insert(0, str(ROOT / "tests"))
    import _inputs
    P = C2["past"]
    q, k, v = _inputs.gqa_case(1, 1, P, C2["query_heads"], C2["kv_heads"], C2["head_dim"],
                               seed=SEED)
    rows = np.ascontiguousarray(k[:, P:P + 1])
    rep = lambda a: np.ascontiguousarray(np.repeat(a, sequences, axis=0))
    return rep(q), rep(rows), rep(k), rep(v)


def cpu_c2_step(oracle, inputs, threads: int) -> float:
    """One C2 step on the host: cacheAppend of the new key and value rows
    (Reference.metal:295-301), then the dense fp64 causal GQA check
    (tests/FlashAttentionTest.mm:53-85) over past + 1 rows.  Returns seconds."""
    import ctypes
    q, rows, k, v = inputs
    n, P, row = q.shape[0], C2["past"], C2["kv_heads"] * C2["head_dim"]
    t0 = time.perf_counter()
    for cache in (k, v):
        oracle.lib().oracle_cache_append(
            ctypes.c_uint(row), ctypes.c_uint(P * row), ctypes.c_uint(n),
            rows.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(row),
            cache.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(cache[0].size))
    oracle.gqa_dense(q, k, v, P, threads=threads)
    return time.perf_counter() - t0


def cpu_op_baselines(budget_s: float = 4.0):
    """Every op of the path on the host cores, all cores and one thread, each on a
    bounded sample of its benchmark config (the CPU baseline table: C1 prefill, C2
    decode step, C3 DeltaNet prefill, C4 DeltaNet step).  Returns {config: entry}."""
    import numpy as np
    sys.path.insert(0, str(ROOT / "tests"))
    import _inputs
    oracle, flags, cores = native_oracle()
    build = f"oracle/oracle.c, gcc {flags} -fopenmp"
    res = {}

    def timed(fn, threads):
        t0 = time.perf_counter()
        fn(threads)
        return time.perf_counter() - t0

    # C1: dense fp64 GQA, B=1, T=128, past 0 (the whole config).
    q, k, v = _inputs.gqa_case(1, 128, 0, 16, 4, 256, seed=SEED)
    flop = 2 * oracle.lib().oracle_gqa_fp_macs(128, 0, 16, 256)
    run = lambda th: oracle.gqa_dense(q, k, v, 0, threads=th)
    run(cores)
    t_all, t_one = timed(run, cores), timed(run, 1)
    res["C1"] = {"unit": "TFLOP/s", "all_cores": round(flop / t_all / 1e12, 6),
                 "one_thread": round(flop / t_one / 1e12, 6), "cores": cores,
                 "sample": f"the whole config; dense fp64 check of FlashAttentionTest.mm:53-85 "
                           f"({build})"}
    # C2: the decode step; all cores on the full batch of 64, one thread on 2 sequences.
    full = c2_host_inputs(C2["batch"])
    cpu_c2_step(oracle, c2_host_inputs(1), cores)
    t_all = cpu_c2_step(oracle, full, cores)
    t_one = cpu_c2_step(oracle, c2_host_inputs(2), 1)
    res["C2"] = {"unit": "GB/s", "all_cores": round(c2_step_bytes(oracle, 64) / t_all / 1e9, 4),
                 "one_thread": round(c2_step_bytes(oracle, 2) / t_one / 1e9, 4), "cores": cores,
                 "sample": f"all cores: the whole step (64 sequences); one thread: 2 sequences; "
                           f"cacheAppend + dense fp64 GQA ({build})"}
    del full
    # C3 and C4: the token-sequential DeltaNet (Graph.metal:146-170 +
    # Reference.metal:182-197).  Bytes of a sample: the cost model's per-sequence
    # bytes of a call of that length.
    def delta_entry(name, tokens_all, seqs_all, tokens_one, seqs_one, std, note):
        out = {"unit": "GB/s", "cores": cores}
        for key, T, B, th in (("all_cores", tokens_all, seqs_all, cores),
                              ("one_thread", tokens_one, seqs_one, 1)):
            c = _inputs.delta_case(B, T, 16, 128, 32, 128, state_std=std, seed=SEED)
            nbytes = sum(oracle.delta_bytes(T, 16, 128, 32, 128)) * B
            secs = timed(lambda th_: oracle.delta_update(c["q"], c["k"], c["v"], c["beta"],
                                                         c["decay"], c["state"], threads=th_), th)
            out[key] = round(nbytes / secs / 1e9, 4)
        out["sample"] = f"{note}; token-sequential DeltaNet ({build})"
        return out

    res["C3"] = delta_entry("C3", 4096, 1, 256, 1, 0.0,
                            "all cores: 1 of the 4 sequences, all 4096 tokens; one thread: 1 "
                            "sequence, 256 tokens")
    res["C4"] = delta_entry("C4", 1, 256, 1, 16, 0.02,
                            "all cores: the whole step (256 sequences); one thread: 16 sequences")
    del np
    return res


# ---------------------------------------------------------------------------
# our arm


def decode_inputs(torch, device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    B, P, CAP = C2["batch"], C2["past"], C2["capacity"]
    Hq, Hkv, D = C2["query_heads"], C2["kv_heads"], C2["head_dim"]
    kc = torch.zeros(B, CAP, Hkv, D, dtype=torch.float16, device=device)
    vc = torch.zeros_like(kc)
    kc[:, :P].normal_(generator=g)
    vc[:, :P].normal_(generator=g)
    q = torch.randn(B, 1, Hq, D, generator=g, device=device).half()
    kn = torch.randn(B, 1, Hkv, D, generator=g, device=device).half()
    vn = torch.randn(B, 1, Hkv, D, generator=g, device=device).half()
    return q, kn, vn, kc, vc


def run_ours(args, dist):
    import torch

    from llminfer_b200 import ops

    device = torch.device("cuda", dist.local)
    torch.cuda.set_device(device)
    peaks = load_peaks()
    P = C2["past"]
    q, kn, vn, kc, vc = decode_inputs(torch, device, SEED + dist.rank)
    kc_bytes = kc.numel() * kc.element_size()
    out = torch.empty_like(q)
    ws = torch.empty(ops.decode_workspace_bytes(C2["batch"], C2["query_heads"], C2["kv_heads"],
                                                C2["head_dim"], P), dtype=torch.uint8,
                     device=device)

    # A decode step as the session lowers it: the KvAppend pair folded into
    # the decode's two kernels (llmi_cuda_gqa_decode_append).  Steps are
    # enqueued back to back on the same caches, so no settled flag.
    def step():
        ops.gqa_decode_append(q, kn, vn, kc, vc, P, out=out, workspace=ws)

    costs = step_bytes([1], 1, P, C2["capacity"], C2["batch"], query_heads=C2["query_heads"],
                       kv_heads=C2["kv_heads"], head_dim=C2["head_dim"])
    bytes_step = costs["KvAppend"][0] + costs["CausalGqa"][0]
    bytes_decode = costs["CausalGqa"][0]

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    K = args.steps
    # The whole-step rate: K steps between two events, nothing recorded in
    # between (an event between two kernels would end the programmatic
    # overlap of their launches).
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch, device) as clocks:
        start.record()
        for i in range(K):
            step()
        end.record()
        torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    # The roofline kernel (gqaScores + gqaSoftmax) alone: a second pass of K
    # steps with events around each decode call.
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(K)]
    for i in range(K):
        ops.cache_append(kn, kc, P)
        ops.cache_append(vn, vc, P)
        ev[i][0].record()
        ops.gqa_decode(q, kc, vc, P, out=out, workspace=ws)
        ev[i][1].record()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    ops.poll_error()
    ms = dist.max(start.elapsed_time(end))
    decode_ms = dist.max(statistics.mean(a.elapsed_time(b) for a, b in ev))
    ms_step = ms / K
    value = bytes_step * dist.world * K / (ms / 1e3) / 1e9
    achieved = bytes_decode / (decode_ms / 1e3) / 1e9
    traffic = profile_traffic("c2_decode", "CausalGqa")

    # End to end through the C-ABI calls with pinned host buffers, pipelined
    # as a serving loop would run it: step i's inputs go up on one copy stream
    # while step i - 1 computes, and each step's output comes back on another;
    # device inputs and outputs are double-buffered.  Every step's copies are
    # inside the timed region (the end event waits for the last read-back).
    hq = torch.empty(q.shape, dtype=q.dtype, pin_memory=True).copy_(q.cpu())
    hk = torch.empty(kn.shape, dtype=kn.dtype, pin_memory=True).copy_(kn.cpu())
    hv = torch.empty(vn.shape, dtype=vn.dtype, pin_memory=True).copy_(vn.cpu())
    hout = [torch.empty(out.shape, dtype=out.dtype, pin_memory=True) for _ in range(2)]
    dq = [torch.empty_like(q) for _ in range(2)]
    dk = [torch.empty_like(kn) for _ in range(2)]
    dv = [torch.empty_like(vn) for _ in range(2)]
    dout = [torch.empty_like(out) for _ in range(2)]
    compute = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    uploaded = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    read_back = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        b = i & 1
        with torch.cuda.stream(up):
            up.wait_event(consumed[b])  # step i - 2 has read buffer b
            dq[b].copy_(hq, non_blocking=True)
            dk[b].copy_(hk, non_blocking=True)
            dv[b].copy_(hv, non_blocking=True)
            uploaded[b].record(up)
        compute.wait_event(uploaded[b])
        compute.wait_event(read_back[b])  # step i - 2's output has left dout[b]
        ops.gqa_decode_append(dq[b], dk[b], dv[b], kc, vc, P, out=dout[b], workspace=ws)
        consumed[b].record(compute)
        with torch.cuda.stream(down):
            down.wait_event(consumed[b])
            hout[b].copy_(dout[b], non_blocking=True)
            read_back[b].record(down)

    for i in range(3):
        e2e_step(i)
    compute.wait_stream(down)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    up.wait_stream(compute)
    down.wait_stream(compute)
    for i in range(K):
        e2e_step(i)
    compute.wait_stream(down)
    e2.record()
    torch.cuda.synchronize()
    dist.barrier()
    e2e_ms = dist.max(s2.elapsed_time(e2))
    h2d = (q.numel() + kn.numel() + vn.numel()) * 2
    d2h = out.numel() * 2

    cpu = None
    cpu_ops = {}
    if not args.no_cpu and dist.world == 1 and dist.rank == 0:
        cpu_ops = cpu_op_baselines()
        c2 = cpu_ops["C2"]
        cpu = {"value": c2["all_cores"], "unit": "GB/s", "cores": c2["cores"], "kind": "port",
               "one_thread_value": c2["one_thread"], "sample": c2["sample"]}

    del q, kn, vn, kc, vc, out, ws, hq, hk, hv, hout, dq, dk, dv, dout
    torch.cuda.empty_cache()
    secondary = []
    if not args.no_secondary:
        secondary = run_secondary(torch, ops, device, peaks, dist)
        for entry in secondary:
            tag = entry["workload"].split(" ")[0]
            if tag in cpu_ops:
                entry["cpu_baseline"] = cpu_ops[tag]
    stack = stack_seq = None
    if not args.no_stack:
        from llminfer_b200.stack import run_stack

        def one_stack(split):
            dist.barrier()
            r = run_stack(torch, dist.pg, dist.world, dist.rank, split=split, **C5)
            r["prefill_frac_of_bf16_peak"] = round(
                r["prefill_tflops"] / dist.world / peaks["bf16_tflops"], 4)
            r["decode_frac_of_hbm_peak"] = round(
                r["decode_gbs"] / dist.world / peaks["hbm_gbs"], 4)
            r["scaling"] = "strong"
            torch.cuda.empty_cache()
            return r

        # The config's (sequence x head) sharding with its all-gathers, and
        # beside it (N > 1) whole sequences per GPU, which needs no collective.
        stack = one_stack("heads")
        if dist.world > 1:
            stack_seq = one_stack("sequences")

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": dist.world,
        "steps": K, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic: seeded N(0,1) fp16 (torch Philox on device), per-rank seed",
        "config": {
            "workload": "C2 GQA decode step (cacheAppend x2 + gqaScores + gqaSoftmax): batch 64 "
                        "per GPU, 1 new token, past 4096, capacity 8192, Hq 16, Hkv 4, D 256, "
                        "fp32 softmax/accumulation",
            "global_batch": C2["batch"] * dist.world, "past": P, "capacity": C2["capacity"],
            "query_heads": C2["query_heads"], "kv_heads": C2["kv_heads"],
            "head_dim": C2["head_dim"],
            "parallelism": f"sequence-sharded over {dist.world} GPU(s), no collective",
            "l2": (f"no flush: each step streams {bytes_step / 1e9:.2f} GB of KV cache rows "
                   f"(the caches hold {2 * kc_bytes / 1e9:.2f} GB at capacity), far above the "
                   f"126 MB L2"),
            "bytes_per_step_per_gpu": bytes_step,
        },
        "roofline": {"kernel": "gqaScores+gqaSoftmax (decode op)", "bound": "hbm",
                     "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                     "peak_source": peaks["source"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic,
                     "algorithmic_bytes_per_launch": bytes_decode,
                     "avg_launch_ms": round(decode_ms, 4)},
        "cpu_baseline": cpu,
        "e2e": {"value": round(bytes_step * dist.world * K / (e2e_ms / 1e3) / 1e9, 2),
                "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms / K, 4),
                "copies": "pinned host buffers; uploads and read-backs on their own streams, "
                          "double-buffered, overlapping the neighbouring steps' kernels"},
        "gpu_launches": 2 * K,
        "clocks": clocks.summary(),
        "secondary": secondary,
        "stack": stack,
        "stack_sequence_major": stack_seq,
    }
    return line


def time_op(torch, fn, dist, reps=10, warmup=3):
    """Median and best CUDA-event time of fn (ms), max over ranks."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(reps)]
    for a, b in evs:
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    t = sorted(a.elapsed_time(b) for a, b in evs)
    return dist.max(statistics.median(t)), dist.max(t[0])


def time_graph(torch, fn, dist, reps=50):
    """Device time per call (ms, max over ranks) of fn captured once into a CUDA graph
    and replayed `reps` times back to back between two events: the GPU-side cost of a
    launch-bound call, without the host's per-call work."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()  # argument checks and one-time set-up outside the capture
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    ms = dist.max(a.elapsed_time(b) / reps)
    del graph
    return ms


def delta_inputs(torch, device, g, B, T, Hk, Hv, state_std, dk=128, dv=128):
    """Seeded DeltaNet operands drawn as the configs say (on the device)."""
    nrm = torch.nn.functional.normalize
    q = (nrm(torch.randn(B, T, Hk, dk, generator=g, device=device), dim=-1) / dk ** 0.5)
    q = q.reshape(B, T, Hk * dk).contiguous()
    k = nrm(torch.randn(B, T, Hk, dk, generator=g, device=device), dim=-1)
    k = k.reshape(B, T, Hk * dk).contiguous()
    v = torch.randn(B, T, Hv * dv, generator=g, device=device).half()
    beta = torch.sigmoid(torch.randn(B, T, Hv, generator=g, device=device)).half().float()
    decay = torch.exp(-torch.nn.functional.softplus(
        torch.randn(B, T, Hv, generator=g, device=device)))
    state = torch.randn(B, Hv, dk, dv, generator=g, device=device) * state_std
    return q, k, v, beta, decay, state


def run_strong(torch, ops, device, peaks, dist, g):
    """C2, C3 and C4 split over the ranks (fixed total work).  Returns one line per
    config: aggregate value (whole job / max-over-ranks time) and, from rank 0's
    run of the whole job on one GPU, the efficiency against 1 GPU."""
    N = dist.world
    out = []

    def replayed_ms(fn, reps):
        """Device time per call of fn replayed from a CUDA graph, back to back (this GPU)."""
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
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
        del graph
        return a.elapsed_time(b) / reps

    def whole_on_one_gpu(make, reps):
        """Rank 0 times the whole job alone on its GPU before any shard runs
        (the other ranks wait at the barrier); returns ms or None."""
        if N == 1:
            return None
        dist.barrier()
        one = None
        if dist.rank == 0:
            fn, _ = make(True)
            one = replayed_ms(fn, reps)
            del fn
        torch.cuda.empty_cache()
        dist.barrier()
        return one

    def line(name, unit_desc, make, total_bytes, reps=20):
        # Each call is replayed from a CUDA graph (as the stack's decode steps
        # are): at a few sequences per GPU a step's kernels take less time than
        # the Python calls that would issue them.
        one = whole_on_one_gpu(make, reps)
        fn, _ = make(False)
        dist.barrier()
        ms = dist.max(replayed_ms(fn, reps))
        del fn
        gbs = total_bytes / (ms / 1e3) / 1e9
        entry = {"workload": name, "scaling": "strong", "split": unit_desc,
                 "ms": round(ms, 4), "value": round(gbs, 1), "unit": "GB/s",
                 "frac_of_hbm_peak_per_gpu": round(gbs / N / peaks["hbm_gbs"], 4),
                 "timing": "CUDA-graph replay, back to back, max over ranks"}
        if N == 1:
            one = ms
        if dist.rank == 0:
            entry["ms_1gpu"] = round(one, 4)
            entry["efficiency_vs_1gpu"] = round(one / (N * ms), 4)
        torch.cuda.empty_cache()
        return entry

    # C2: the decode step (two appends + decode) of 64 sequences.
    P, CAP = C2["past"], C2["capacity"]
    Hq, Hkv, D = C2["query_heads"], C2["kv_heads"], C2["head_dim"]
    per_seq = step_bytes([1], 1, P, CAP, 1, query_heads=Hq, kv_heads=Hkv, head_dim=D)
    seq_bytes = per_seq["KvAppend"][0] + per_seq["CausalGqa"][0]

    def make_c2(whole):
        B = 64 if whole else 64 // N
        kc = torch.zeros(B, CAP, Hkv, D, dtype=torch.float16, device=device)
        vc = torch.zeros_like(kc)
        kc[:, :P].normal_(generator=g)
        vc[:, :P].normal_(generator=g)
        q = torch.randn(B, 1, Hq, D, generator=g, device=device).half()
        kn = torch.randn(B, 1, Hkv, D, generator=g, device=device).half()
        o = torch.empty_like(q)
        ws = torch.empty(ops.decode_workspace_bytes(B, Hq, Hkv, D, P), dtype=torch.uint8,
                         device=device)

        # KvAppend folded into the decode, with settled cache rows, as the
        # session issues a decode step: every replay is its own graph launch,
        # so the rows [0, P) it reads are complete before it starts.
        def fn():
            ops.gqa_decode_append(q, kn, kn, kc, vc, P, out=o, workspace=ws, settled=True)
        return fn, seq_bytes * B

    out.append(line("C2 GQA decode step, 64 sequences in all (cacheAppend x2 + gqaScores + "
                    "gqaSoftmax, the appends folded into the decode's kernels)",
                    f"{64 // N} sequences per GPU", make_c2, seq_bytes * 64))

    # C3: DeltaNet prefill, B=4, T=4096, 128 (sequence, value head) units.
    B3, T3 = 4, 4096
    cost3 = step_bytes([0], T3, 0, T3, B3, key_heads=16, key_dim=128, value_heads=32,
                       value_dim=128)["DeltaUpdate"]

    def make_c3(whole):
        Hk, Hv = (16, 32) if whole else (16 // N, 32 // N)
        q, k, v, beta, decay, state = delta_inputs(torch, device, g, B3, T3, Hk, Hv, 0.0)
        o = torch.empty_like(v)
        ws = torch.empty(max(16, ops.delta_workspace_bytes(B3, T3, Hk, 128, Hv, 128)),
                         dtype=torch.uint8, device=device)
        return (lambda: ops.delta_update(q, k, v, beta, decay, state, out=o, workspace=ws)), 0

    out.append(line("C3 DeltaNet prefill B=4 T=4096, 128 (sequence, value head) units in all "
                    "(graphDeltaUpdate, chunked)",
                    f"{128 // N} units per GPU: 4 sequences x {32 // N} value heads "
                    f"({16 // N} key heads)", make_c3, cost3[0], reps=10))
    out[-1]["tflops_cost_model"] = round(2 * cost3[1] / (out[-1]["ms"] / 1e3) / 1e12, 3)

    # C4: DeltaNet recurrent step, 256 sequences.
    cost4 = step_bytes([0], 1, 0, 1, 256, key_heads=16, key_dim=128, value_heads=32,
                       value_dim=128)["DeltaUpdate"]

    def make_c4(whole):
        B = 256 if whole else 256 // N
        q, k, v, beta, decay, state = delta_inputs(torch, device, g, B, 1, 16, 32, 0.02)
        o = torch.empty_like(v)
        ws = torch.empty(16, dtype=torch.uint8, device=device)  # one token takes no scratch
        # Settled state: each replay is its own graph launch.
        return (lambda: ops.delta_update(q, k, v, beta, decay, state, out=o, workspace=ws,
                                         settled=True)), 0

    out.append(line("C4 DeltaNet recurrent step, 256 sequences in all (graphDeltaUpdate)",
                    f"{256 // N} sequences per GPU", make_c4, cost4[0]))
    return out


def time_abi_calls(torch, ops, q, kc, vc, out, dist, reps=200):
    """Per-call time of llmi_cuda_gqa_prefill called straight through ctypes with its
    arguments prepared once, `reps` calls back to back between two events: the C
    entry point's host cost (checks, cached tensor maps, launch) where it exceeds
    the kernel's device time."""
    import ctypes
    abi = ops.abi
    p = abi.GqaParams(q.shape[1], q.shape[2], kc.shape[2], q.shape[3], 0)
    args = (ctypes.byref(p), q.shape[0], q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
            kc.stride(0), out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    call = abi.lib.llmi_cuda_gqa_prefill
    for _ in range(10):
        abi.check(call(*args))
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        call(*args)
    b.record()
    torch.cuda.synchronize()
    return dist.max(a.elapsed_time(b) / reps)


def run_secondary(torch, ops, device, peaks, dist):
    """The other kernels of the path on their benchmark configs (CUDA events, median,
    max over ranks).  Every rank runs the whole config on its own GPU, so with N GPUs
    the aggregate is N times the per-GPU work over the slowest rank's time."""
    g = torch.Generator(device=device)
    g.manual_seed(SEED + dist.rank)
    N = dist.world
    res = []
    # C2, C3 and C4 as fixed jobs split over the N GPUs (strong scaling):
    # C2's 64 sequences, C3's 128 (sequence, value head) units as groups of
    # whole key heads, C4's 256 sequences.  Each rank times its shard; rank 0
    # also times the whole job alone on its GPU, which gives the efficiency
    # t(1 GPU) / (N t(N GPUs)).  They run first: the long tensor-core prefill
    # below leaves the GPU under its power cap for a while afterwards.
    res.extend(run_strong(torch, ops, device, peaks, dist, g))
    # C1: GQA prefill, B=1, T=128, past 0.
    q = torch.randn(1, 128, 16, 256, generator=g, device=device).half()
    kc = torch.randn(1, 128, 4, 256, generator=g, device=device).half()
    vc = torch.randn(1, 128, 4, 256, generator=g, device=device).half()
    out = torch.empty_like(q)
    med, best = time_op(torch, lambda: ops.gqa_prefill(q, kc, vc, 0, out=out), dist)
    graph_ms = time_graph(torch, lambda: ops.gqa_prefill(q, kc, vc, 0, out=out), dist)
    abi_ms = time_abi_calls(torch, ops, q, kc, vc, out, dist)
    macs = step_bytes([1], 128, 0, 128, 1, query_heads=16, kv_heads=4, head_dim=256)["CausalGqa"][1]
    tf = 2 * macs / (med / 1e3) / 1e12
    tf_graph = 2 * macs / (graph_ms / 1e3) / 1e12
    res.append({"workload": "C1 GQA prefill B=1 T=128 past 0 (gqaFlashAttention)"
                            + (f", {N} replicas" if N > 1 else ""),
                "ms": round(med, 4), "value": round(tf * N, 3), "unit": "TFLOP/s",
                "frac_of_bf16_peak": round(tf / peaks["bf16_tflops"], 4),
                # Launch-bound: the same call captured in a CUDA graph and replayed,
                # and the C-ABI call alone issued back to back (no Python wrapper).
                "graph_replay_ms": round(graph_ms, 4), "graph_replay_value": round(tf_graph * N, 3),
                "c_abi_call_ms": round(abi_ms, 4)})
    del q, kc, vc, out
    # Producers at the C5 layer shapes (B=16 per GPU, T=8192): q/k RmsNorm +
    # partial RoPE of a GQA layer (k into the cache), and a DeltaNet layer's
    # conv + SiLU + q/k L2 norm and gates.  Bytes: each operand read and
    # written once.
    B, T, D = 16, 8192, 256
    Hk, dk, Hv, dv = 16, 128, 32, 128
    qg = torch.randn(B, T, 16, 2 * D, generator=g, device=device).half()
    kr = torch.randn(B, T, 4, D, generator=g, device=device).half()
    wq = (0.1 * torch.randn(D, generator=g, device=device)).float()
    wk = (0.1 * torch.randn(D, generator=g, device=device)).float()
    qo = torch.empty(B, T, 16, D, dtype=torch.float16, device=device)
    cache = torch.empty(B, T, 4, D, dtype=torch.float16, device=device)

    def rope():
        ops.norm_rope(qg, wq, 0, D // 4, 1e7, head_dim=D, out=qo)
        ops.norm_rope(kr, wk, 0, D // 4, 1e7, out=cache, output_start=0)

    med, best = time_op(torch, rope, dist, reps=5, warmup=2)
    gbs = 2 * (qo.numel() + cache.numel()) * 2 / (med / 1e3) / 1e9
    res.append({"workload": "q/k RmsNorm + partial RoPE of a GQA layer, k into the cache, "
                            "C5 shape B=16 T=8192 per GPU (normRope)",
                "ms": round(med, 4), "value": round(gbs * N, 1), "unit": "GB/s",
                "frac_of_hbm_peak": round(gbs / peaks["hbm_gbs"], 4)})
    del qg, kr, qo, cache
    W = 2 * Hk * dk + Hv * dv
    qkv = torch.randn(B, T, W, generator=g, device=device).half()
    wconv = (0.5 * torch.randn(W, 4, generator=g, device=device)).half()
    hist = torch.zeros(B, W, 3, dtype=torch.float16, device=device)
    ga = torch.randn(B, T, Hv, generator=g, device=device).half()
    gb = torch.randn(B, T, Hv, generator=g, device=device).half()
    a_log = torch.randn(Hv, generator=g, device=device).float()
    dt_bias = torch.randn(Hv, generator=g, device=device).float()

    def prep():
        ops.delta_prepare(qkv, wconv, hist, Hk, dk, Hv, dv)
        ops.delta_gates(ga, gb, a_log, dt_bias)

    med, best = time_op(torch, prep, dist, reps=5, warmup=2)
    nbytes = B * T * (W * 2 + 2 * Hk * dk * 4 + Hv * dv * 2 + Hv * (2 * 2 + 2 * 4))
    gbs = nbytes / (med / 1e3) / 1e9
    res.append({"workload": "DeltaNet layer inputs: conv + SiLU + q/k L2 norm and gates, "
                            "C5 shape B=16 T=8192 per GPU (deltaPrepare, deltaGates)",
                "ms": round(med, 4), "value": round(gbs * N, 1), "unit": "GB/s",
                "frac_of_hbm_peak": round(gbs / peaks["hbm_gbs"], 4)})
    # The GQA prefill at one C5 layer's shape: B=16 (per GPU), T=8192, past 0.
    # Measured last: at the power cap it leaves the next few milliseconds of
    # work on the GPU slower.
    # Each launch is ~6 ms and the loop runs under the power cap, so the
    # sustained peak is the denominator that applies; burst is given too.
    B, T = 16, 8192
    q = torch.randn(B, T, 16, 256, generator=g, device=device).half()
    kc = torch.randn(B, T, 4, 256, generator=g, device=device).half()
    vc = torch.randn(B, T, 4, 256, generator=g, device=device).half()
    out = torch.empty_like(q)
    med, best = time_op(torch, lambda: ops.gqa_prefill(q, kc, vc, 0, out=out), dist, reps=5,
                        warmup=2)
    macs = step_bytes([1], T, 0, T, B, query_heads=16, kv_heads=4, head_dim=256)["CausalGqa"][1]
    tf = 2 * macs / (med / 1e3) / 1e12
    res.append({"workload": "GQA prefill at the C5 layer shape: B=16 per GPU, T=8192, past 0 "
                            "(gqaFlashAttention)",
                "ms": round(med, 4), "value": round(tf * N, 1), "unit": "TFLOP/s",
                "frac_of_bf16_peak": round(tf / peaks["bf16_tflops"], 4),
                "frac_of_bf16_sustained": round(tf / peaks["bf16_tflops_sustained"], 4)})
    del q, kc, vc, out
    return res


# ---------------------------------------------------------------------------
# reference arm


def run_reference(args):
    """The reference arm: the reference's scalar check code for the C2 step, restated in
    oracle/ (the reference's own path is Metal and cannot run here), on every host core.
    Each timed step is the whole C2 step (64 sequences), the same work at every N; under
    torchrun only rank 0 runs it, the other ranks exit without work."""
    if int(os.environ.get("RANK", "0")) != 0:
        return None
    oracle, flags, cores = native_oracle()
    full = c2_host_inputs(C2["batch"])
    for _ in range(max(args.warmup, 1)):
        cpu_c2_step(oracle, full, cores)
    times = [cpu_c2_step(oracle, full, cores) for _ in range(args.steps)]
    secs = sum(times)
    value = c2_step_bytes(oracle, C2["batch"]) * args.steps / secs / 1e9
    one_secs = cpu_c2_step(oracle, c2_host_inputs(2), 1)
    one_value = c2_step_bytes(oracle, 2) / one_secs / 1e9
    sample = (f"each step the whole C2 step: cacheAppend of the new rows and the dense fp64 "
              f"causal GQA of all 64 sequences (tests/FlashAttentionTest.mm:53-85, "
              f"Reference.metal:295-301 restated in oracle/oracle.c, gcc {flags} -fopenmp, "
              f"{cores} threads); the reference's own path is Metal and cannot run here")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    return {
        "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "impl": "reference",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(secs / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic: seeded N(0,1) fp16 (numpy Philox)",
        "config": {"workload": "C2 GQA decode step (cacheAppend x2 + causal GQA): batch 64, "
                               "1 new token, past 4096, Hq 16, Hkv 4, D 256",
                   "global_batch": C2["batch"], "past": C2["past"], "capacity": C2["capacity"],
                   "query_heads": C2["query_heads"], "kv_heads": C2["kv_heads"],
                   "head_dim": C2["head_dim"], "parallelism": f"host cores (OpenMP, {cores})"},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": cores,
                         "kind": "port", "sample": sample},
        "cpu_one_thread": {"value": round(one_value, 4), "unit": "GB/s", "cores": 1,
                           "sample": "2 sequences of the C2 step on one thread"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }


def main():
    args = parse_args()
    # Only the JSON line goes to stdout: libraries that print at start-up
    # (NCCL's version banner, for one) are sent to stderr.
    result_out = os.fdopen(os.dup(sys.stdout.fileno()), "w")
    sys.stdout.flush()
    os.dup2(sys.stderr.fileno(), sys.stdout.fileno())
    if args.impl == "reference":
        # No process group and no GPU work: rank 0 times the host cores, the
        # other ranks exit at once.
        line = run_reference(args)
        if line is not None:
            print(json.dumps(line), file=result_out, flush=True)
        return
    dist = Dist(args.gpus)
    try:
        line = run_ours(args, dist)
        if dist.rank == 0 and line is not None:
            print(json.dumps(line), file=result_out, flush=True)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
