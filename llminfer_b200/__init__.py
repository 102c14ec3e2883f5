"""B200 (sm_100a) CUDA backend for llminfer's attention hot path.

The product is the C-ABI library llminfer_b200/_lib/libllmi_cuda.so
(include/llmi_cuda.h): GQA flash attention (causal prefill, split-K decode
against the KV cache, cacheAppend) and the Gated-DeltaNet update (recurrent
step and chunked prefill), plus the attention-stack session that owns the
KV caches and recurrent states and lowers each step's ops with the
reference's --plan kernel names.  This package binds it for Python callers.
The bindings load on first use, and fail loudly without the built library
(there is no fallback); the build module itself (`python -m
llminfer_b200.build`) needs no library.
"""
import importlib

__all__ = ["abi", "LlmiError", "describe_step", "make_stack_config", "ops"]


def __getattr__(name):
    # The library and torch load lazily: host-only users (plan description)
    # do not pay for torch, and the build runs with a stale or missing library.
    if name in ("abi", "LlmiError", "describe_step", "make_stack_config"):
        abi = importlib.import_module("._abi", __name__)
        return abi if name == "abi" else getattr(abi, name)
    if name == "ops":
        return importlib.import_module(".ops", __name__)
    raise AttributeError(name)
