"""ctypes binding of the C ABI in include/llmi_cuda.h.

The library is llminfer_b200/_lib/libllmi_cuda.so, built in-tree by
llminfer_b200/build.py.  Importing this module without the library raises
ImportError: there is no fallback implementation of any op.
"""
from __future__ import annotations

import ctypes
from ctypes import (POINTER, c_char_p, c_float, c_int, c_size_t, c_ubyte, c_uint, c_uint16, c_uint64,
                    c_void_p)
from pathlib import Path

LIBRARY_PATH = Path(__file__).resolve().parent / "_lib" / "libllmi_cuda.so"

LLMI_OK = 0
LLMI_INVALID_ARGUMENT = 1
LLMI_UNSUPPORTED = 2
LLMI_CUDA_ERROR = 3
LLMI_DEVICE_TIMEOUT = 4
LLMI_WORKSPACE_TOO_SMALL = 5
LLMI_SESSION_INVALID = 6
LLMI_CAPACITY_EXCEEDED = 7

LLMI_FLAG_SETTLED = 1  # launch flag of the _ex entry points (include/llmi_cuda.h)

LAYER_DELTANET = 0
LAYER_GQA = 1

STATE_KEYS = 0
STATE_VALUES = 1
STATE_RECURRENT = 2
STATE_CONV_HISTORY = 3


class CacheParams(ctypes.Structure):
    """CacheParams of lib/Backend/Metal/Kernels/ReferenceParams.h:49-51."""
    _fields_ = [("count", c_uint), ("offset", c_uint)]


class GqaParams(ctypes.Structure):
    """GqaParams of lib/Backend/Metal/Kernels/ReferenceParams.h:53-55."""
    _fields_ = [("tokens", c_uint), ("queryHeads", c_uint), ("kvHeads", c_uint),
                ("headDim", c_uint), ("past", c_uint)]


class DeltaParams(ctypes.Structure):
    """GraphDeltaParams of lib/Backend/Metal/Kernels/GraphParams.h:50-52."""
    _fields_ = [("tokens", c_uint), ("keyHeads", c_uint), ("keyDim", c_uint),
                ("valueHeads", c_uint), ("valueDim", c_uint)]


class RopeParams(ctypes.Structure):
    """RopeParams of lib/Backend/Metal/Kernels/ReferenceParams.h:44-47."""
    _fields_ = [(n, c_uint) for n in ("tokens", "heads", "headDim", "rotaryDim", "headStride",
                                      "past", "outputStart")] + \
               [("epsilon", c_float), ("theta", c_float)]


class ConvParams(ctypes.Structure):
    """ConvParams of lib/Backend/Metal/Kernels/ReferenceParams.h:32-34."""
    _fields_ = [(n, c_uint) for n in ("tokens", "channels", "kernelSize", "applySilu")]


class L2Params(ctypes.Structure):
    """L2Params of lib/Backend/Metal/Kernels/GraphParams.h:30-33."""
    _fields_ = [("rows", c_uint), ("width", c_uint), ("epsilon", c_float), ("scale", c_float)]


class RowParams(ctypes.Structure):
    """RowParams of lib/Backend/Metal/Kernels/ReferenceParams.h:23-26."""
    _fields_ = [("rows", c_uint), ("width", c_uint), ("epsilon", c_float)]


class DeltaPrepParams(ctypes.Structure):
    """DeltaParams of ReferenceParams.h:40-42 plus the conv size and L2 epsilon."""
    _fields_ = [(n, c_uint) for n in ("tokens", "keyHeads", "keyDim", "valueHeads", "valueDim",
                                      "qkvWidth", "kernelSize")] + [("epsilon", c_float)]


class StackConfig(ctypes.Structure):
    _fields_ = [("layers", c_uint), ("layer_kinds", POINTER(c_ubyte)),
                ("batch", c_uint), ("capacity", c_uint),
                ("queryHeads", c_uint), ("kvHeads", c_uint), ("headDim", c_uint),
                ("keyHeads", c_uint), ("keyDim", c_uint), ("valueHeads", c_uint),
                ("valueDim", c_uint)]


class LayerIO(ctypes.Structure):
    _fields_ = [("q", c_void_p), ("k", c_void_p), ("v", c_void_p),
                ("beta", c_void_p), ("decay", c_void_p), ("out", c_void_p)]


class ProducerConfig(ctypes.Structure):
    _fields_ = [("rotaryDim", c_uint), ("ropeTheta", c_float), ("normEpsilon", c_float),
                ("convKernel", c_uint), ("l2Epsilon", c_float)]


class LayerProjections(ctypes.Structure):
    _fields_ = [("qg", c_void_p), ("k", c_void_p), ("v", c_void_p),
                ("qNorm", c_void_p), ("kNorm", c_void_p),
                ("qkv", c_void_p), ("a", c_void_p), ("b", c_void_p), ("convWeight", c_void_p),
                ("aLog", c_void_p), ("dtBias", c_void_p), ("out", c_void_p)]


# (name, restype, argtypes) of every exported entry point, in header order.
SIGNATURES = [
    ("llmi_cuda_last_error", c_char_p, []),
    ("llmi_cuda_status_name", c_char_p, [c_int]),
    ("llmi_cuda_cache_append", c_int,
     [POINTER(CacheParams), c_uint, c_void_p, c_size_t, c_void_p, c_size_t, c_void_p]),
    ("llmi_cuda_gqa_prefill", c_int,
     [POINTER(GqaParams), c_uint, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    ("llmi_cuda_gqa_decode_workspace", c_size_t, [POINTER(GqaParams), c_uint]),
    ("llmi_cuda_gqa_decode", c_int,
     [POINTER(GqaParams), c_uint, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p,
      c_void_p, c_size_t, c_void_p]),
    ("llmi_cuda_gqa_decode_append", c_int,
     [POINTER(GqaParams), c_uint, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p,
      c_size_t, c_void_p, c_void_p, c_size_t, c_void_p]),
    ("llmi_cuda_gqa_decode_append_ex", c_int,
     [POINTER(GqaParams), c_uint, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p,
      c_size_t, c_void_p, c_void_p, c_size_t, c_void_p, c_uint]),
    ("llmi_cuda_gqa_decode_noalloc", c_int,
     [POINTER(GqaParams), c_uint, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    ("llmi_cuda_delta_update", c_int,
     [POINTER(DeltaParams), c_uint, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
      c_void_p, c_void_p, c_void_p]),
    ("llmi_cuda_delta_update_workspace", c_size_t, [POINTER(DeltaParams), c_uint]),
    ("llmi_cuda_delta_update_ws", c_int,
     [POINTER(DeltaParams), c_uint, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
      c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    ("llmi_cuda_delta_update_ws_ex", c_int,
     [POINTER(DeltaParams), c_uint, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
      c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_uint]),
    ("llmi_cuda_norm_rope", c_int,
     [POINTER(RopeParams), c_uint, c_void_p, c_size_t, c_void_p, c_void_p, c_size_t, c_void_p]),
    ("llmi_cuda_partial_rope", c_int,
     [POINTER(RopeParams), c_uint, c_void_p, c_size_t, c_void_p, c_size_t, c_void_p]),
    ("llmi_cuda_causal_conv", c_int,
     [POINTER(ConvParams), c_uint, c_void_p, c_size_t, c_void_p, c_void_p, c_size_t, c_void_p,
      c_size_t, c_void_p]),
    ("llmi_cuda_l2_norm", c_int, [POINTER(L2Params), c_void_p, c_void_p, c_void_p]),
    ("llmi_cuda_delta_gates", c_int,
     [POINTER(RowParams), c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    ("llmi_cuda_delta_prepare", c_int,
     [POINTER(DeltaPrepParams), c_uint, c_void_p, c_size_t, c_void_p, c_void_p, c_size_t,
      c_void_p, c_void_p, c_void_p, c_void_p]),
    ("llmi_cuda_poll_error", c_int, [c_void_p]),
    ("llmi_cuda_selftest_wait_timeout", c_int, [c_uint, c_void_p]),
    ("llmi_cuda_session_open", c_int, [POINTER(StackConfig), c_void_p, POINTER(c_void_p)]),
    ("llmi_cuda_session_close", None, [c_void_p]),
    ("llmi_cuda_session_step", c_int, [c_void_p, c_uint, POINTER(LayerIO), c_int]),
    ("llmi_cuda_session_enqueue", c_int, [c_void_p, c_uint, POINTER(LayerIO)]),
    ("llmi_cuda_session_sync", c_int, [c_void_p]),
    ("llmi_cuda_session_set_layer_events", c_int, [c_void_p, POINTER(c_void_p), c_uint]),
    ("llmi_cuda_session_inject_fault", c_int, [c_void_p, c_uint]),
    ("llmi_cuda_session_reset", c_int, [c_void_p]),
    ("llmi_cuda_session_past", c_uint64, [c_void_p]),
    ("llmi_cuda_session_is_invalid", c_int, [c_void_p]),
    ("llmi_cuda_session_state", c_int,
     [c_void_p, c_uint, c_uint, POINTER(c_void_p), POINTER(c_size_t)]),
    ("llmi_cuda_session_read_state", c_int, [c_void_p, c_uint, c_uint, c_void_p, c_size_t]),
    ("llmi_cuda_session_write_state", c_int, [c_void_p, c_uint, c_uint, c_void_p, c_size_t]),
    ("llmi_cuda_session_set_producers", c_int, [c_void_p, POINTER(ProducerConfig)]),
    ("llmi_cuda_session_step_projections", c_int,
     [c_void_p, c_uint, POINTER(LayerProjections), c_int]),
    ("llmi_cuda_session_plan", c_size_t, [c_void_p, c_char_p, c_size_t]),
    ("llmi_cuda_describe_step", c_size_t,
     [POINTER(StackConfig), c_uint, c_uint64, c_char_p, c_size_t, POINTER(c_int)]),
]


def _load() -> ctypes.CDLL:
    if not LIBRARY_PATH.exists():
        raise ImportError(
            f"{LIBRARY_PATH} is missing: build it with `python -m llminfer_b200.build` "
            "(or __graft_entry__.build()); there is no non-CUDA implementation")
    lib = ctypes.CDLL(str(LIBRARY_PATH))
    for name, restype, argtypes in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


lib = _load()


class LlmiError(RuntimeError):
    """A non-zero llmi_status from the CUDA backend."""

    def __init__(self, status: int, message: str):
        self.status = status
        name = lib.llmi_cuda_status_name(status).decode()
        super().__init__(f"{name}: {message}")


def check(status: int) -> None:
    if status != LLMI_OK:
        raise LlmiError(status, lib.llmi_cuda_last_error().decode())


def make_stack_config(kinds, batch, capacity, query_heads=0, kv_heads=0, head_dim=0,
                      key_heads=0, key_dim=0, value_heads=0, value_dim=0):
    """Returns (StackConfig, keep-alive array) for a list of LAYER_* kinds."""
    array = (c_ubyte * len(kinds))(*kinds)
    cfg = StackConfig(len(kinds), ctypes.cast(array, POINTER(c_ubyte)), batch, capacity,
                      query_heads, kv_heads, head_dim, key_heads, key_dim, value_heads, value_dim)
    return cfg, array


def describe_step(cfg: StackConfig, tokens: int, past: int) -> str:
    """Host-only lowering of one step (no GPU): JSON text."""
    status = c_int(0)
    need = lib.llmi_cuda_describe_step(ctypes.byref(cfg), tokens, past, None, 0,
                                       ctypes.byref(status))
    check(status.value)
    buf = ctypes.create_string_buffer(need + 1)
    lib.llmi_cuda_describe_step(ctypes.byref(cfg), tokens, past, buf, need + 1,
                                ctypes.byref(status))
    check(status.value)
    return buf.value.decode()


__all__ = [n for n in dir() if not n.startswith("_")] + ["c_uint16"]
