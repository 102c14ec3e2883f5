"""torch-facing wrappers of the C ABI (include/llmi_cuda.h).

PyTorch only provides device memory and streams here; every op runs the CUDA
kernels of libllmi_cuda.so.  Shapes follow the reference's operands with a
leading sequence (batch) dimension:

  GQA       q, out        [B, T, Hq, D]       fp16
            k/v cache     [B, capacity, Hkv, D] fp16
  DeltaNet  q, k          [B, T, Hk*dk]       fp32
            v, out        [B, T, Hv*dv]       fp16
            beta, decay   [B, T, Hv]          fp32
            state         [B, Hv, dk, dv]     fp32 (updated in place)
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _abi as abi
from ._abi import LlmiError, check, lib


def _stream(stream: torch.cuda.Stream | None) -> int:
    s = torch.cuda.current_stream() if stream is None else stream
    return s.cuda_stream


def _need(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous CUDA {dtype} tensor "
                         f"(got {t.dtype} on {t.device}, contiguous={t.is_contiguous()})")


def cache_append(rows: torch.Tensor, cache: torch.Tensor, past: int,
                 stream: torch.cuda.Stream | None = None) -> None:
    """cacheAppend: writes rows [B, T, Hkv, D] into cache [B, cap, Hkv, D] at [past, past+T)."""
    _need(rows, torch.float16, "rows")
    _need(cache, torch.float16, "cache")
    B, T, H, D = rows.shape
    if cache.shape[0] != B or cache.shape[2:] != (H, D) or past + T > cache.shape[1]:
        raise ValueError("cache_append: rows do not fit the cache")
    row = H * D
    p = abi.CacheParams(T * row, past * row)
    check(lib.llmi_cuda_cache_append(ctypes.byref(p), B, rows.data_ptr(), T * row,
                                     cache.data_ptr(), cache.shape[1] * row, _stream(stream)))


def _gqa_params(q, k_cache, past):
    B, T, Hq, D = q.shape
    if k_cache.shape[0] != B or k_cache.shape[3] != D:
        raise ValueError("q and cache shapes disagree")
    return abi.GqaParams(T, Hq, k_cache.shape[2], D, past)


def gqa_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, past: int,
                out: torch.Tensor | None = None,
                stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """gqaFlashAttention over cache rows [0, past+T) (T >= 1)."""
    for t, n in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _need(t, torch.float16, n)
    p = _gqa_params(q, k_cache, past)
    out = torch.empty_like(q) if out is None else out
    _need(out, torch.float16, "out")
    stride = k_cache.stride(0)
    check(lib.llmi_cuda_gqa_prefill(ctypes.byref(p), q.shape[0], q.data_ptr(),
                                    k_cache.data_ptr(), v_cache.data_ptr(), stride,
                                    out.data_ptr(), _stream(stream)))
    return out


def decode_workspace_bytes(batch: int, query_heads: int, kv_heads: int, head_dim: int,
                           past: int) -> int:
    p = abi.GqaParams(1, query_heads, kv_heads, head_dim, past)
    n = lib.llmi_cuda_gqa_decode_workspace(ctypes.byref(p), batch)
    if n == 0:
        raise LlmiError(abi.LLMI_CUDA_ERROR, lib.llmi_cuda_last_error().decode())
    return n


def gqa_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, past: int,
               out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
               stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """gqaScores + gqaSoftmax: one query token per sequence over cache rows [0, past+1)."""
    for t, n in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _need(t, torch.float16, n)
    p = _gqa_params(q, k_cache, past)
    if workspace is None:
        n = decode_workspace_bytes(q.shape[0], p.queryHeads, p.kvHeads, p.headDim, past)
        workspace = torch.empty(n, dtype=torch.uint8, device=q.device)
    out = torch.empty_like(q) if out is None else out
    _need(out, torch.float16, "out")
    stride = k_cache.stride(0)
    check(lib.llmi_cuda_gqa_decode(ctypes.byref(p), q.shape[0], q.data_ptr(),
                                   k_cache.data_ptr(), v_cache.data_ptr(), stride,
                                   out.data_ptr(), workspace.data_ptr(), workspace.numel(),
                                   _stream(stream)))
    return out


def gqa_decode_append(q: torch.Tensor, k_new: torch.Tensor | None, v_new: torch.Tensor | None,
                      k_cache: torch.Tensor, v_cache: torch.Tensor, past: int,
                      out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                      stream: torch.cuda.Stream | None = None,
                      settled: bool = False) -> torch.Tensor:
    """KvAppend + decode in one pass: writes k_new / v_new [B, 1, Hkv, D] (None: that
    row is already in the cache) into cache row `past`, then decodes over rows
    [0, past] like gqa_decode.

    settled=True passes LLMI_FLAG_SETTLED: the caller guarantees that no work
    still running when the call starts writes cache rows [0, past) (the stream
    was synchronised after the last write, or the write belongs to an earlier
    CUDA graph launch).  Same results; the kernels read those rows before the
    kernel ahead has finished."""
    for t, n in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _need(t, torch.float16, n)
    p = _gqa_params(q, k_cache, past)
    row = p.kvHeads * p.headDim
    new_stride = 0
    for t, n in ((k_new, "k_new"), (v_new, "v_new")):
        if t is None:
            continue
        _need(t, torch.float16, n)
        if t.shape != (q.shape[0], 1, p.kvHeads, p.headDim):
            raise ValueError(f"{n} must be [B, 1, Hkv, D]")
        if new_stride and t.stride(0) != new_stride:
            raise ValueError("k_new and v_new must share one sequence stride")
        new_stride = t.stride(0)
    if past + 1 > k_cache.shape[1]:
        raise ValueError("gqa_decode_append: the cache is full")
    if workspace is None:
        n = decode_workspace_bytes(q.shape[0], p.queryHeads, p.kvHeads, p.headDim, past)
        workspace = torch.empty(n, dtype=torch.uint8, device=q.device)
    out = torch.empty_like(q) if out is None else out
    _need(out, torch.float16, "out")
    check(lib.llmi_cuda_gqa_decode_append_ex(
        ctypes.byref(p), q.shape[0], q.data_ptr(),
        k_new.data_ptr() if k_new is not None else None,
        v_new.data_ptr() if v_new is not None else None, new_stride or row,
        k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0), out.data_ptr(),
        workspace.data_ptr(), workspace.numel(), _stream(stream),
        abi.LLMI_FLAG_SETTLED if settled else 0))
    return out


def delta_workspace_bytes(batch: int, tokens: int, key_heads: int, key_dim: int,
                          value_heads: int, value_dim: int) -> int:
    """Scratch bytes of delta_update's chunk-parallel form (0 if the call does not use it)."""
    p = abi.DeltaParams(tokens, key_heads, key_dim, value_heads, value_dim)
    return lib.llmi_cuda_delta_update_workspace(ctypes.byref(p), batch)


def delta_update(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
                 decay: torch.Tensor, state: torch.Tensor, out: torch.Tensor | None = None,
                 workspace: torch.Tensor | bool | None = None,
                 stream: torch.cuda.Stream | None = None,
                 settled: bool = False) -> torch.Tensor:
    """graphDeltaUpdate: updates state [B, Hv, dk, dv] in place, returns out [B, T, Hv*dv].

    workspace None allocates the scratch of the chunk-parallel form
    (llmi_cuda_delta_update_ws); a uint8 tensor is used as that scratch;
    False calls llmi_cuda_delta_update, which takes no scratch (one kernel
    walks each head's chunks and solves their systems in order).
    settled=True (not with workspace=False) passes LLMI_FLAG_SETTLED, with the
    guarantee gqa_decode_append states, for the state."""
    for t, n in ((q, "q"), (k, "k"), (beta, "beta"), (decay, "decay"), (state, "state")):
        _need(t, torch.float32, n)
    _need(v, torch.float16, "v")
    B, T, key_width = q.shape
    _, Hv, dk, dv = state.shape
    p = abi.DeltaParams(T, key_width // dk, dk, Hv, dv)
    out = torch.empty_like(v) if out is None else out
    _need(out, torch.float16, "out")
    if workspace is False:
        if settled:
            raise ValueError("delta_update: settled needs the workspace entry point")
        check(lib.llmi_cuda_delta_update(ctypes.byref(p), B, q.data_ptr(), k.data_ptr(),
                                         v.data_ptr(), beta.data_ptr(), decay.data_ptr(),
                                         state.data_ptr(), out.data_ptr(), _stream(stream)))
        return out
    if workspace is None:
        n = lib.llmi_cuda_delta_update_workspace(ctypes.byref(p), B)
        workspace = torch.empty(max(n, 16), dtype=torch.uint8, device=q.device)
    check(lib.llmi_cuda_delta_update_ws_ex(ctypes.byref(p), B, q.data_ptr(), k.data_ptr(),
                                           v.data_ptr(), beta.data_ptr(), decay.data_ptr(),
                                           state.data_ptr(), out.data_ptr(),
                                           workspace.data_ptr(), workspace.numel(),
                                           _stream(stream),
                                           abi.LLMI_FLAG_SETTLED if settled else 0))
    return out


# ---- producers of the path's operands --------------------------------------------


def norm_rope(x: torch.Tensor, weight: torch.Tensor | None, past: int, rotary_dim: int,
              theta: float, eps: float = 1e-6, head_dim: int | None = None,
              out: torch.Tensor | None = None, output_start: int = 0,
              stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """normRope (weight given) or partialRope (weight None) over x [B, T, H, W]
    fp16, whose rows are the first head_dim of each W-wide head.  Writes
    rows output_start.. of `out` [B, rows, H, head_dim] (a key cache, with
    output_start = past) or a new [B, T, H, head_dim] tensor."""
    _need(x, torch.float16, "x")
    B, T, H, W = x.shape
    head_dim = head_dim or W
    if out is None:
        out = torch.empty(B, T, H, head_dim, dtype=torch.float16, device=x.device)
    _need(out, torch.float16, "out")
    p = abi.RopeParams(T, H, head_dim, rotary_dim, W, past, output_start, eps, theta)
    if weight is None:
        check(lib.llmi_cuda_partial_rope(ctypes.byref(p), B, x.data_ptr(), x[0].numel(),
                                         out.data_ptr(), out[0].numel(), _stream(stream)))
    else:
        _need(weight, torch.float32, "weight")
        check(lib.llmi_cuda_norm_rope(ctypes.byref(p), B, x.data_ptr(), x[0].numel(),
                                      weight.data_ptr(), out.data_ptr(), out[0].numel(),
                                      _stream(stream)))
    return out


def causal_conv(x: torch.Tensor, weight: torch.Tensor, history: torch.Tensor,
                apply_silu: bool = False, out: torch.Tensor | None = None,
                stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """causalConv over x [B, T, C] fp16 with weight [C, K] and history
    [B, C, K-1] (advanced in place)."""
    for t, n in ((x, "x"), (weight, "weight"), (history, "history")):
        _need(t, torch.float16, n)
    B, T, C = x.shape
    out = torch.empty_like(x) if out is None else out
    p = abi.ConvParams(T, C, weight.shape[1], 1 if apply_silu else 0)
    check(lib.llmi_cuda_causal_conv(ctypes.byref(p), B, x.data_ptr(), x[0].numel(),
                                    weight.data_ptr(), history.data_ptr(), history[0].numel(),
                                    out.data_ptr(), out[0].numel(), _stream(stream)))
    return out


def l2_norm(x: torch.Tensor, width: int, scale: float, eps: float = 1e-6,
            stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """l2NormF32: fp16 rows of `width` -> fp32."""
    _need(x, torch.float16, "x")
    out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    p = abi.L2Params(x.numel() // width, width, eps, scale)
    check(lib.llmi_cuda_l2_norm(ctypes.byref(p), x.data_ptr(), out.data_ptr(), _stream(stream)))
    return out


def delta_gates(a: torch.Tensor, b: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor,
                stream: torch.cuda.Stream | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """deltaGates: a, b [..., H] fp16 -> (beta, decay) fp32."""
    _need(a, torch.float16, "a")
    _need(b, torch.float16, "b")
    _need(a_log, torch.float32, "a_log")
    _need(dt_bias, torch.float32, "dt_bias")
    heads = a.shape[-1]
    beta = torch.empty(a.shape, dtype=torch.float32, device=a.device)
    decay = torch.empty_like(beta)
    p = abi.RowParams(a.numel() // heads, heads, 0.0)
    check(lib.llmi_cuda_delta_gates(ctypes.byref(p), a.data_ptr(), b.data_ptr(),
                                    a_log.data_ptr(), dt_bias.data_ptr(), beta.data_ptr(),
                                    decay.data_ptr(), _stream(stream)))
    return beta, decay


def delta_prepare(qkv: torch.Tensor, conv_weight: torch.Tensor, history: torch.Tensor,
                  key_heads: int, key_dim: int, value_heads: int, value_dim: int,
                  eps: float = 1e-6, stream: torch.cuda.Stream | None = None):
    """The DeltaNet block's (q, k, v) from its qkv projection [B, T, W] fp16:
    conv + SiLU, Slices, q/k L2Norm.  Advances history [B, W, K-1] in place."""
    for t, n in ((qkv, "qkv"), (conv_weight, "conv_weight"), (history, "history")):
        _need(t, torch.float16, n)
    B, T, W = qkv.shape
    kw, vw = key_heads * key_dim, value_heads * value_dim
    q = torch.empty(B, T, kw, dtype=torch.float32, device=qkv.device)
    k = torch.empty_like(q)
    v = torch.empty(B, T, vw, dtype=torch.float16, device=qkv.device)
    p = abi.DeltaPrepParams(T, key_heads, key_dim, value_heads, value_dim, W,
                            conv_weight.shape[1], eps)
    check(lib.llmi_cuda_delta_prepare(ctypes.byref(p), B, qkv.data_ptr(), qkv[0].numel(),
                                      conv_weight.data_ptr(), history.data_ptr(),
                                      history[0].numel(), q.data_ptr(), k.data_ptr(),
                                      v.data_ptr(), _stream(stream)))
    return q, k, v


def poll_error(stream: torch.cuda.Stream | None = None) -> None:
    check(lib.llmi_cuda_poll_error(_stream(stream)))


def selftest_wait_timeout(limit_us: int = 1000, stream: torch.cuda.Stream | None = None) -> None:
    """Launches the bounded-wait self-test; the next poll_error raises LLMI_DEVICE_TIMEOUT."""
    check(lib.llmi_cuda_selftest_wait_timeout(limit_us, _stream(stream)))


@dataclass
class LayerTensors:
    """One layer's step operands (see LayerIO in llmi_cuda.h)."""
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    out: torch.Tensor
    beta: torch.Tensor | None = None
    decay: torch.Tensor | None = None

    def to_abi(self) -> abi.LayerIO:
        ptr = lambda t: None if t is None else t.data_ptr()
        return abi.LayerIO(ptr(self.q), ptr(self.k), ptr(self.v), ptr(self.beta),
                           ptr(self.decay), ptr(self.out))


@dataclass
class LayerProjections:
    """One layer's projection outputs and weights (see llmi_layer_projections in
    llmi_cuda.h).  GQA layers: qg, k, v, q_norm, k_norm, out; DeltaNet layers: qkv,
    a, b, conv_weight, a_log, dt_bias, out."""
    out: torch.Tensor
    qg: torch.Tensor | None = None
    k: torch.Tensor | None = None
    v: torch.Tensor | None = None
    q_norm: torch.Tensor | None = None
    k_norm: torch.Tensor | None = None
    qkv: torch.Tensor | None = None
    a: torch.Tensor | None = None
    b: torch.Tensor | None = None
    conv_weight: torch.Tensor | None = None
    a_log: torch.Tensor | None = None
    dt_bias: torch.Tensor | None = None

    def to_abi(self) -> abi.LayerProjections:
        ptr = lambda t: None if t is None else t.data_ptr()
        return abi.LayerProjections(ptr(self.qg), ptr(self.k), ptr(self.v), ptr(self.q_norm),
                                    ptr(self.k_norm), ptr(self.qkv), ptr(self.a), ptr(self.b),
                                    ptr(self.conv_weight), ptr(self.a_log), ptr(self.dt_bias),
                                    ptr(self.out))


class AttentionSession:
    """The attention-stack session (llmi_cuda_session_*), a MetalSession for the attention ops."""

    def __init__(self, kinds, batch, capacity, query_heads=0, kv_heads=0, head_dim=0,
                 key_heads=0, key_dim=0, value_heads=0, value_dim=0,
                 stream: torch.cuda.Stream | None = None):
        self.kinds = list(kinds)
        self.batch, self.capacity = batch, capacity
        self.shape = dict(query_heads=query_heads, kv_heads=kv_heads, head_dim=head_dim,
                          key_heads=key_heads, key_dim=key_dim, value_heads=value_heads,
                          value_dim=value_dim)
        self.stream = torch.cuda.Stream() if stream is None else stream
        self._cfg, self._kinds = abi.make_stack_config(self.kinds, batch, capacity, query_heads,
                                                       kv_heads, head_dim, key_heads, key_dim,
                                                       value_heads, value_dim)
        handle = ctypes.c_void_p()
        check(lib.llmi_cuda_session_open(ctypes.byref(self._cfg), self.stream.cuda_stream,
                                         ctypes.byref(handle)))
        self._handle = handle

    def close(self) -> None:
        if getattr(self, "_handle", None):
            lib.llmi_cuda_session_close(self._handle)
            self._handle = None

    def __del__(self):
        self.close()

    def _io(self, layers):
        if len(layers) != len(self.kinds):
            raise ValueError(f"{len(layers)} layer operand sets for {len(self.kinds)} layers")
        return (abi.LayerIO * len(layers))(*[x.to_abi() for x in layers])

    def step(self, tokens: int, layers, trace_plan: bool = False) -> None:
        self._sync_inputs()
        check(lib.llmi_cuda_session_step(self._handle, tokens, self._io(layers), int(trace_plan)))

    def set_producers(self, rotary_dim: int = 64, rope_theta: float = 10_000_000.0,
                      norm_epsilon: float = 1e-6, conv_kernel: int = 4,
                      l2_epsilon: float = 1e-6) -> None:
        """Enable step_projections (llmi_cuda_session_set_producers)."""
        self._producers = abi.ProducerConfig(rotary_dim, rope_theta, norm_epsilon, conv_kernel,
                                             l2_epsilon)
        check(lib.llmi_cuda_session_set_producers(self._handle, ctypes.byref(self._producers)))

    def step_projections(self, tokens: int, layers, trace_plan: bool = False) -> None:
        """A step from the layers' projection outputs (a list of LayerProjections)."""
        if len(layers) != len(self.kinds):
            raise ValueError(f"{len(layers)} layer operand sets for {len(self.kinds)} layers")
        self._sync_inputs()
        table = (abi.LayerProjections * len(layers))(*[x.to_abi() for x in layers])
        check(lib.llmi_cuda_session_step_projections(self._handle, tokens, table,
                                                      int(trace_plan)))

    def operand_table(self, layers):
        """The C operand table (llmi_layer_io[]) of `layers`.  It holds raw device
        pointers: reusable for every step over the same buffers while they live."""
        return self._io(layers)

    def enqueue(self, tokens: int, layers) -> None:
        """Enqueue a step; `layers` is a list of LayerTensors or an operand_table()."""
        table = layers if isinstance(layers, ctypes.Array) else self._io(layers)
        check(lib.llmi_cuda_session_enqueue(self._handle, tokens, table))

    def sync(self) -> None:
        check(lib.llmi_cuda_session_sync(self._handle))

    def reset(self) -> None:
        check(lib.llmi_cuda_session_reset(self._handle))

    def inject_fault(self, limit_us: int = 1000) -> None:
        """The next step also runs the bounded-wait self-test, so it fails with
        LLMI_DEVICE_TIMEOUT and the session becomes invalid until reset."""
        check(lib.llmi_cuda_session_inject_fault(self._handle, limit_us))

    def set_layer_events(self, events) -> None:
        """Record events[l] on the session stream after layer l of every step
        (None clears).  Events must already exist (recorded once)."""
        if events is None:
            check(lib.llmi_cuda_session_set_layer_events(self._handle, None, 0))
            self._layer_events = None
            return
        handles = (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])
        check(lib.llmi_cuda_session_set_layer_events(self._handle, handles, len(events)))
        self._layer_events = list(events)  # keep them alive while registered

    def _sync_inputs(self) -> None:
        # Operands produced on torch's current stream must be ready before the
        # session stream reads them.
        self.stream.wait_stream(torch.cuda.current_stream())

    @property
    def past(self) -> int:
        return lib.llmi_cuda_session_past(self._handle)

    @property
    def invalid(self) -> bool:
        return bool(lib.llmi_cuda_session_is_invalid(self._handle))

    def plan(self) -> list[dict]:
        import json
        n = lib.llmi_cuda_session_plan(self._handle, None, 0)
        buf = ctypes.create_string_buffer(n + 1)
        lib.llmi_cuda_session_plan(self._handle, buf, n + 1)
        return [json.loads(line) for line in buf.value.decode().splitlines() if line]

    def _state_shape(self, which: int):
        s = self.shape
        if which == abi.STATE_RECURRENT:
            return (self.batch, s["value_heads"], s["key_dim"], s["value_dim"]), torch.float32
        if which == abi.STATE_CONV_HISTORY:
            width = 2 * s["key_heads"] * s["key_dim"] + s["value_heads"] * s["value_dim"]
            return (self.batch, width, self._producers.convKernel - 1), torch.float16
        return (self.batch, self.capacity, s["kv_heads"], s["head_dim"]), torch.float16

    def read_state(self, layer: int, which: int) -> torch.Tensor:
        shape, dtype = self._state_shape(which)
        t = torch.empty(shape, dtype=dtype, device="cuda")
        torch.cuda.current_stream().synchronize()
        check(lib.llmi_cuda_session_read_state(self._handle, layer, which, t.data_ptr(),
                                               t.numel() * t.element_size()))
        return t

    def write_state(self, layer: int, which: int, value: torch.Tensor) -> None:
        shape, dtype = self._state_shape(which)
        value = value.to(device="cuda", dtype=dtype).contiguous().reshape(shape)
        torch.cuda.current_stream().synchronize()
        check(lib.llmi_cuda_session_write_state(self._handle, layer, which, value.data_ptr(),
                                                value.numel() * value.element_size()))
