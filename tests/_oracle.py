"""ctypes loader of the CPU oracle (oracle/build/liboracle.so) for tests.

The oracle is the checker: tests compare the CUDA results against it.  It is
built on first use with `make -C oracle` when missing.
"""
from __future__ import annotations

import ctypes
import subprocess
from ctypes import POINTER, c_double, c_float, c_int, c_size_t, c_uint, c_uint16, c_uint32, c_uint64
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
ORACLE_DIR = ROOT / "oracle"
LIB_PATH = ORACLE_DIR / "build" / "liboracle.so"
REF_PATH = ORACLE_DIR / "_ref" / "libllmi_ref.so"


class GqaParams(ctypes.Structure):
    _fields_ = [("tokens", c_uint), ("queryHeads", c_uint), ("kvHeads", c_uint),
                ("headDim", c_uint), ("past", c_uint)]


class DeltaParams(ctypes.Structure):
    _fields_ = [("tokens", c_uint), ("keyHeads", c_uint), ("keyDim", c_uint),
                ("valueHeads", c_uint), ("valueDim", c_uint)]


class RopeParams(ctypes.Structure):
    _fields_ = [(n, c_uint) for n in ("tokens", "heads", "headDim", "rotaryDim", "headStride",
                                      "past", "outputStart")] + \
               [("epsilon", c_float), ("theta", c_float)]


class ConvParams(ctypes.Structure):
    _fields_ = [(n, c_uint) for n in ("tokens", "channels", "kernelSize", "applySilu")]


def _ptr(a: np.ndarray, ctype):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(POINTER(ctype))


def load(path: Path | None = None) -> ctypes.CDLL:
    path = LIB_PATH if path is None else path
    if not path.exists():
        subprocess.run(["make", "-C", str(ORACLE_DIR)], check=True, capture_output=True)
    lib = ctypes.CDLL(str(path))
    lib.oracle_f32_to_f16.restype = c_uint16
    lib.oracle_f32_to_f16.argtypes = [c_float]
    lib.oracle_f16_to_f32.restype = c_float
    lib.oracle_f16_to_f32.argtypes = [c_uint16]
    lib.oracle_max_threads.restype = c_int
    for name in ("oracle_gqa_pairs",):
        getattr(lib, name).restype = c_uint64
        getattr(lib, name).argtypes = [c_uint64, c_uint64]
    lib.oracle_gqa_fp_macs.restype = c_uint64
    lib.oracle_gqa_fp_macs.argtypes = [c_uint64] * 4
    lib.oracle_delta_fp_macs.restype = c_uint64
    lib.oracle_delta_fp_macs.argtypes = [c_uint64] * 4
    lib.oracle_kv_append_bytes.argtypes = [c_uint64] * 3 + [POINTER(c_uint64)] * 2
    lib.oracle_gqa_bytes.argtypes = [c_uint64] * 5 + [POINTER(c_uint64)] * 2
    lib.oracle_delta_bytes.argtypes = [c_uint64] * 5 + [POINTER(c_uint64)] * 2
    lib.oracle_set_threads.argtypes = [c_int]
    return lib


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = load()
    return _lib


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_f32_to_f16_array(_ptr(x, c_float), _ptr(out, c_uint16), c_size_t(x.size))
    return out


def f16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().oracle_f16_to_f32_array(_ptr(h, c_uint16), _ptr(out, c_float), c_size_t(h.size))
    return out


def lcg_fill(state: int, n: int) -> tuple[np.ndarray, int]:
    """FlashAttentionTest.mm's LCG fill; returns (fp16 bits, next state)."""
    s = c_uint32(state)
    out = np.empty(n, dtype=np.uint16)
    lib().oracle_lcg_fill(ctypes.byref(s), _ptr(out, c_uint16), c_size_t(n))
    return out, s.value


def _as_bits(a: np.ndarray) -> np.ndarray:
    if a.dtype == np.float16:
        return np.ascontiguousarray(a).view(np.uint16)
    assert a.dtype == np.uint16
    return np.ascontiguousarray(a)


def gqa_dense(q, k_cache, v_cache, past: int, threads: int = 0) -> np.ndarray:
    """fp64 dense causal GQA.  q [B,T,Hq,D], caches [B,rows,Hkv,D] (fp16 or bits)."""
    q, k, v = _as_bits(q), _as_bits(k_cache), _as_bits(v_cache)
    B, T, Hq, D = q.shape
    p = GqaParams(T, Hq, k.shape[2], D, past)
    out = np.empty((B, T, Hq, D), dtype=np.float64)
    lib().oracle_gqa_dense(ctypes.byref(p), c_uint(B), _ptr(q, c_uint16), c_size_t(T * Hq * D),
                           _ptr(k, c_uint16), _ptr(v, c_uint16), c_size_t(k[0].size),
                           _ptr(out, c_double), c_int(threads))
    return out


def gqa_dense_rows(q_rows, k_seq, v_seq, past: int, tokens: int, query_heads: int,
                   token, head, threads: int = 0) -> np.ndarray:
    """fp64 dense causal GQA of chosen rows of one sequence.  q_rows [n,D] are
    the rows (token[i], head[i]); k_seq/v_seq [rows,Hkv,D] that sequence's
    cache.  Returns [n,D] float64."""
    q, k, v = _as_bits(q_rows), _as_bits(k_seq), _as_bits(v_seq)
    n, D = q.shape
    token = np.ascontiguousarray(token, np.uint32)
    head = np.ascontiguousarray(head, np.uint32)
    p = GqaParams(tokens, query_heads, k.shape[1], D, past)
    out = np.empty((n, D), dtype=np.float64)
    lib().oracle_gqa_dense_rows(ctypes.byref(p), _ptr(q, c_uint16), _ptr(k, c_uint16),
                                _ptr(v, c_uint16), _ptr(token, c_uint), _ptr(head, c_uint),
                                c_uint(n), _ptr(out, c_double), c_int(threads))
    return out


def gqa_eager_f16(q, k_cache, v_cache, past: int, threads: int = 0) -> np.ndarray:
    """The reference decode path with its fp16 rounding points; returns float16."""
    q, k, v = _as_bits(q), _as_bits(k_cache), _as_bits(v_cache)
    B, T, Hq, D = q.shape
    p = GqaParams(T, Hq, k.shape[2], D, past)
    out = np.empty((B, T, Hq, D), dtype=np.uint16)
    lib().oracle_gqa_eager_f16(ctypes.byref(p), c_uint(B), _ptr(q, c_uint16),
                               c_size_t(T * Hq * D), _ptr(k, c_uint16), _ptr(v, c_uint16),
                               c_size_t(k[0].size), _ptr(out, c_uint16), c_int(threads))
    return out.view(np.float16)


def delta_update(q, k, v, beta, decay, state, threads: int = 0):
    """Token-sequential DeltaNet.  Returns (out float16 [B,T,Hv*dv], new state)."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = _as_bits(v)
    beta = np.ascontiguousarray(beta, np.float32)
    decay = np.ascontiguousarray(decay, np.float32)
    state = np.array(state, dtype=np.float32, order="C", copy=True)
    B, Hv, dk, dv = state.shape
    T = q.shape[1]
    Hk = q.shape[2] // dk
    p = DeltaParams(T, Hk, dk, Hv, dv)
    out = np.empty((B, T, Hv * dv), dtype=np.uint16)
    lib().oracle_delta_update(ctypes.byref(p), c_uint(B), _ptr(q, c_float), _ptr(k, c_float),
                              _ptr(v, c_uint16), _ptr(beta, c_float), _ptr(decay, c_float),
                              _ptr(state, c_float), _ptr(out, c_uint16), c_int(threads))
    return out.view(np.float16), state


def l2norm(x: np.ndarray, width: int, scale: float, eps: float = 1e-6) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().oracle_l2norm(_ptr(x, c_float), _ptr(out, c_float), c_size_t(x.size // width),
                        c_uint(width), c_float(eps), c_float(scale))
    return out


def delta_gates(a: np.ndarray, b: np.ndarray, a_log: np.ndarray, dt_bias: np.ndarray):
    """deltaGates on fp16 inputs a, b [rows][heads] -> (beta, decay) fp32."""
    af = f16_bits_to_f32(_as_bits(a))
    bf = f16_bits_to_f32(_as_bits(b))
    heads = af.shape[-1]
    beta = np.empty(af.shape, np.float32)
    decay = np.empty(af.shape, np.float32)
    a_log = np.ascontiguousarray(a_log, np.float32)
    dt_bias = np.ascontiguousarray(dt_bias, np.float32)
    lib().oracle_delta_gates(_ptr(af, c_float), _ptr(bf, c_float), _ptr(a_log, c_float),
                             _ptr(dt_bias, c_float), c_size_t(af.size // heads), c_uint(heads),
                             _ptr(beta, c_float), _ptr(decay, c_float))
    return beta, decay


def norm_rope(x: np.ndarray, weight, past: int, rotary_dim: int, theta: float,
              eps: float = 1e-6, head_dim: int | None = None, output=None, output_start: int = 0):
    """normRope / partialRope over x [batch][tokens][heads][width] fp16 (the
    row is the first head_dim of each width-wide head); weight None skips the
    norm.  Writes rows output_start.. of `output` [batch][rows][heads][head_dim]
    (a copy is returned), or a fresh [batch][tokens][heads][head_dim] array."""
    x = np.ascontiguousarray(_as_bits(x))
    batch, tokens, heads, width = x.shape
    head_dim = head_dim or width
    if output is None:
        out = np.zeros((batch, tokens, heads, head_dim), np.uint16)
    else:
        out = np.ascontiguousarray(_as_bits(output)).copy()
    p = RopeParams(tokens, heads, head_dim, rotary_dim, width, past, output_start, eps, theta)
    w = None if weight is None else np.ascontiguousarray(weight, np.float32)
    lib().oracle_norm_rope(ctypes.byref(p), c_uint(batch), _ptr(x, c_uint16),
                           c_size_t(x[0].size), None if w is None else _ptr(w, c_float),
                           _ptr(out, c_uint16), c_size_t(out[0].size))
    return out.view(np.float16)


def causal_conv(x: np.ndarray, weight: np.ndarray, history: np.ndarray, apply_silu: bool):
    """causalConv over x [batch][tokens][channels] fp16 with weight
    [channels][kernel] fp16 and history [batch][channels][kernel-1] fp16.
    Returns (out fp16, the advanced history)."""
    x = np.ascontiguousarray(_as_bits(x))
    w = np.ascontiguousarray(_as_bits(weight))
    hist = np.ascontiguousarray(_as_bits(history)).copy()
    batch, tokens, channels = x.shape
    out = np.empty_like(x)
    p = ConvParams(tokens, channels, w.shape[1], 1 if apply_silu else 0)
    lib().oracle_causal_conv(ctypes.byref(p), c_uint(batch), _ptr(x, c_uint16),
                             c_size_t(x[0].size), _ptr(w, c_uint16), _ptr(hist, c_uint16),
                             c_size_t(hist[0].size), _ptr(out, c_uint16), c_size_t(out[0].size))
    return out.view(np.float16), hist.view(np.float16)


def delta_prepare(qkv, weight, history, key_heads, key_dim, value_heads, value_dim, eps=1e-6):
    """The DeltaNet block's q, k (fp32) and v (fp16) from its qkv projection:
    causalConv with SiLU, the Slices, l2NormF32 of q (scale 1/sqrt(keyDim))
    and k (scale 1) (Qwen35ModelBuilder.cpp:146-157).  Returns (q, k, v,
    advanced history)."""
    conv, hist = causal_conv(qkv, weight, history, True)
    kw = key_heads * key_dim
    cf = f16_bits_to_f32(conv.view(np.uint16))
    q = l2norm(cf[..., :kw], key_dim, 1.0 / np.sqrt(np.float32(key_dim)), eps)
    k = l2norm(cf[..., kw:2 * kw], key_dim, 1.0, eps)
    v = np.ascontiguousarray(conv[..., 2 * kw:2 * kw + value_heads * value_dim])
    return q, k, v, hist


def reference_shim():
    """The reference's own GraphIR/cost/fp16 code (oracle/_ref), or None."""
    if not REF_PATH.exists():
        return None
    ref = ctypes.CDLL(str(REF_PATH))
    ref.ref_float_to_half.restype = c_uint16
    ref.ref_float_to_half.argtypes = [c_float]
    ref.ref_half_to_float.restype = c_float
    ref.ref_half_to_float.argtypes = [c_uint16]
    ref.ref_field_count.restype = c_int
    ref.ref_attention_costs.restype = c_int
    ref.ref_attention_costs.argtypes = [c_uint64] * 10 + [POINTER(c_uint64)]
    return ref


def _bytes(fn, *args) -> tuple[int, int]:
    r, w = c_uint64(), c_uint64()
    fn(*args, ctypes.byref(r), ctypes.byref(w))
    return r.value, w.value


def kv_append_bytes(tokens, kv_heads, head_dim) -> tuple[int, int]:
    """(read, write) logical bytes of one sequence's KvAppend (Cost.cpp:85-93)."""
    return _bytes(lib().oracle_kv_append_bytes, tokens, kv_heads, head_dim)


def gqa_bytes(tokens, past, query_heads, kv_heads, head_dim) -> tuple[int, int]:
    """(read, write) logical bytes of one sequence's CausalGqa."""
    return _bytes(lib().oracle_gqa_bytes, tokens, past, query_heads, kv_heads, head_dim)


def delta_bytes(tokens, key_heads, key_dim, value_heads, value_dim) -> tuple[int, int]:
    """(read, write) logical bytes of one sequence's DeltaUpdate."""
    return _bytes(lib().oracle_delta_bytes, tokens, key_heads, key_dim, value_heads, value_dim)
