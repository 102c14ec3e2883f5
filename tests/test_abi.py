"""C-ABI and host-logic tests that need no GPU.

* the library loads and exports every entry point include/llmi_cuda.h declares;
* the host op verifier and cost model agree with the reference's own GraphIR
  (values computed by its compiled C++, tests/golden/reference_pins.json) and
  with the pins of tests/GraphIRTest.cpp and tests/ConverterTest.py;
* the lowering reports the reference's --plan kernel names
  (tests/MetalReferenceTest.py:458-472: flash iff the chunk has more than one
  token, otherwise gqaScores and gqaSoftmax);
* argument errors are reported before anything touches a device.
"""
import ctypes
import json
import re
from pathlib import Path

import pytest

import llminfer_b200 as L
from llminfer_b200 import abi

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"


def declared_symbols():
    text = (ROOT / "include" / "llmi_cuda.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(llmi_cuda_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    names = declared_symbols()
    assert len(names) >= 20
    for name in names:
        assert hasattr(abi.lib, name), name
    bound = {n for n, _, _ in abi.SIGNATURES}
    assert bound == set(names), set(names) ^ bound


def test_status_names():
    assert abi.lib.llmi_cuda_status_name(abi.LLMI_UNSUPPORTED) == b"LLMI_UNSUPPORTED"
    assert abi.lib.llmi_cuda_status_name(99) == b"LLMI_UNKNOWN_STATUS"


def describe(kinds, tokens, past, capacity, batch=1, **shape):
    cfg, keep = L.make_stack_config(kinds, batch, capacity, **shape)
    return json.loads(L.describe_step(cfg, tokens, past))


def test_graphir_pins():
    # tests/GraphIRTest.cpp:74-104 and tests/ConverterTest.py:170-187: T=3,
    # P=2, capacity 8, 2 query heads / 1 kv head of 8, DeltaNet 2 value heads
    # of 4 x 4 (1 key head).
    d = describe([0, 1], 3, 2, 8, query_heads=2, kv_heads=1, head_dim=8,
                 key_heads=1, key_dim=4, value_heads=2, value_dim=4)
    delta, kv, gqa = d["ops"]
    assert [o["kind"] for o in d["ops"]] == ["DeltaUpdate", "KvAppend", "CausalGqa"]
    assert kv["cost"]["logical_write_bytes"] == 96
    assert gqa["cost"]["logical_read_bytes"] == 256
    assert gqa["cost"]["fp_macs"] == 384
    assert delta["cost"]["fp_macs"] == 288
    assert all(e["begin"] == 2 and e["length"] == 3 and e["version_before"] == 0
               and e["version_after"] == 1 for e in kv["effects"])
    assert all(e["begin"] == 0 and e["length"] == 5 and e["version_before"] == 1
               and e["version_after"] == 1 for e in gqa["effects"])


def test_costs_and_effects_match_reference_graphir():
    pins = json.loads((GOLDEN / "reference_pins.json").read_text())["attention_costs"]
    fields = pins["fields"]
    checked = 0
    for case in pins["cases"]:
        tokens, past, capacity = case["step"]
        hq, hkv, d, hk, dk, hv, dv = case["shape"]
        cfg, keep = L.make_stack_config([1, 0], 1, capacity, hq, hkv, d, hk, dk, hv, dv)
        if case["status"] != 0:
            with pytest.raises(L.LlmiError):
                L.describe_step(cfg, tokens, past)
            continue
        got = json.loads(L.describe_step(cfg, tokens, past))
        kv, gqa, delta = got["ops"]
        want = dict(zip(fields, case["record"]))
        assert kv["cost"]["logical_write_bytes"] == want["kv_write_bytes"]
        assert (kv["effects"][0]["begin"], kv["effects"][0]["length"]) == (want["kv_begin"], want["kv_length"])
        assert (kv["effects"][0]["version_before"], kv["effects"][0]["version_after"]) == (
            want["kv_version_before"], want["kv_version_after"])
        assert gqa["cost"]["logical_read_bytes"] == want["gqa_read_bytes"]
        assert gqa["cost"]["logical_write_bytes"] == want["gqa_write_bytes"]
        assert gqa["cost"]["fp_macs"] == want["gqa_fp_macs"]
        assert (gqa["effects"][0]["begin"], gqa["effects"][0]["length"]) == (want["gqa_begin"], want["gqa_length"])
        assert (gqa["effects"][0]["version_before"], gqa["effects"][0]["version_after"]) == (
            want["gqa_version_before"], want["gqa_version_after"])
        assert delta["cost"]["logical_read_bytes"] == want["delta_read_bytes"]
        assert delta["cost"]["logical_write_bytes"] == want["delta_write_bytes"]
        assert delta["cost"]["fp_macs"] == want["delta_fp_macs"]
        checked += 1
    assert checked >= 20


@pytest.mark.parametrize("tokens,past", [(1, 0), (1, 4096), (2, 0), (17, 5), (128, 0)])
def test_plan_names_follow_the_reference_lowering(tokens, past):
    kinds = [0, 0, 0, 1] * 2  # the 3:1 DeltaNet:GQA interleave of Qwen3.5
    d = describe(kinds, tokens, past, 8192, batch=4, query_heads=16, kv_heads=4, head_dim=256,
                 key_heads=16, key_dim=128, value_heads=32, value_dim=128)
    kernels = [x["kernel"] for x in d["dispatches"]]
    indices = [x["op_index"] for x in d["dispatches"]]
    assert indices == sorted(indices)
    assert set(indices) == set(range(len(d["ops"])))
    flash = tokens > 1
    assert ("gqaFlashAttention" in kernels) == flash
    assert ("gqaScores" in kernels) != flash
    assert ("gqaSoftmax" in kernels) != flash
    assert kernels.count("cacheAppend") == 2 * kinds.count(1)
    assert kernels.count("graphDeltaUpdate") == kinds.count(0)
    for op in d["ops"]:
        names = [x["kernel"] for x in d["dispatches"] if x["op_index"] == op["index"]]
        if op["kind"] == "KvAppend":
            assert names == ["cacheAppend", "cacheAppend"]
        elif op["kind"] == "CausalGqa":
            assert names == (["gqaFlashAttention"] if flash else ["gqaScores", "gqaSoftmax"])
        else:
            assert names == ["graphDeltaUpdate"]


@pytest.mark.parametrize("tokens,past,capacity", [(0, 0, 8), (9, 0, 8), (2, 7, 8), (1, 9, 8)])
def test_invalid_steps_are_rejected(tokens, past, capacity):
    cfg, keep = L.make_stack_config([1], 1, capacity, 2, 1, 8)
    with pytest.raises(L.LlmiError) as err:
        L.describe_step(cfg, tokens, past)
    assert err.value.status == abi.LLMI_CAPACITY_EXCEEDED


def test_invalid_configs_are_rejected():
    for kinds, shape in [([1], dict(query_heads=3, kv_heads=2, head_dim=8)),
                         ([0], dict(key_heads=3, key_dim=4, value_heads=4, value_dim=4)),
                         ([5], dict())]:
        cfg, keep = L.make_stack_config(kinds, 1, 8, **shape)
        with pytest.raises(L.LlmiError) as err:
            L.describe_step(cfg, 1, 0)
        assert err.value.status == abi.LLMI_INVALID_ARGUMENT


def test_argument_errors_precede_any_device_use():
    lib = abi.lib
    g = abi.GqaParams(1, 16, 4, 256, 0)
    assert lib.llmi_cuda_gqa_prefill(ctypes.byref(g), 1, None, None, None, 0, None, None) == abi.LLMI_INVALID_ARGUMENT
    assert lib.llmi_cuda_gqa_decode(ctypes.byref(g), 1, None, None, None, 0, None, None, 0, None) == abi.LLMI_INVALID_ARGUMENT
    bad = abi.GqaParams(1, 6, 4, 256, 0)
    one = ctypes.c_void_p(16)
    assert lib.llmi_cuda_gqa_prefill(ctypes.byref(bad), 1, one, one, one, 1 << 20, one, None) == abi.LLMI_INVALID_ARGUMENT
    d = abi.DeltaParams(1, 16, 128, 32, 128)
    assert lib.llmi_cuda_delta_update(ctypes.byref(d), 1, None, None, None, None, None, None, None, None) == abi.LLMI_INVALID_ARGUMENT
    c = abi.CacheParams(8, 0)
    assert lib.llmi_cuda_cache_append(ctypes.byref(c), 0, one, 8, one, 8, None) == abi.LLMI_INVALID_ARGUMENT
    assert "null" in lib.llmi_cuda_last_error().decode() or "zero" in lib.llmi_cuda_last_error().decode()


def test_unknown_launch_flags_are_rejected_before_any_device_use():
    lib = abi.lib
    one = ctypes.c_void_p(16)
    g = abi.GqaParams(1, 16, 4, 256, 7)
    status = lib.llmi_cuda_gqa_decode_append_ex(ctypes.byref(g), 1, one, one, one, 1024, one, one,
                                                1 << 20, one, one, 1 << 20, None, 2)
    assert status == abi.LLMI_INVALID_ARGUMENT
    assert "flags" in lib.llmi_cuda_last_error().decode()
    d = abi.DeltaParams(1, 16, 128, 32, 128)
    status = lib.llmi_cuda_delta_update_ws_ex(ctypes.byref(d), 1, one, one, one, one, one, one,
                                              one, one, 16, None, abi.LLMI_FLAG_SETTLED | 4)
    assert status == abi.LLMI_INVALID_ARGUMENT
    assert "flags" in lib.llmi_cuda_last_error().decode()
