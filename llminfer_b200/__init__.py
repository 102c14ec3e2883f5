"""B200 (sm_100a) CUDA backend for llminfer's attention hot path.

The product is the C-ABI library llminfer_b200/_lib/libllmi_cuda.so
(include/llmi_cuda.h): GQA flash attention (causal prefill, split-K decode
against the KV cache, cacheAppend) and the Gated-DeltaNet update (recurrent
step and chunked prefill), plus the attention-stack session that owns the
KV caches and recurrent states and lowers each step's ops with the
reference's --plan kernel names.  This package binds it for Python callers;
importing it without the built library fails (there is no fallback).
"""
from ._abi import LlmiError, describe_step, make_stack_config  # noqa: F401
from . import _abi as abi  # noqa: F401

__all__ = ["abi", "LlmiError", "describe_step", "make_stack_config", "ops"]


def __getattr__(name):
    # torch is imported lazily so host-only users (plan description) do not
    # pay for it.
    if name == "ops":
        import importlib
        return importlib.import_module(".ops", __name__)
    raise AttributeError(name)
