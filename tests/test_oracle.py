"""Pins of the CPU oracle (oracle/oracle.c) — run without a GPU.

The reference implements this path only as Metal kernels, which cannot run
here, so the oracle is pinned against everything the reference offers that
does run:
  * its own C++ fp16 conversion (floatToHalf / halfToFloat,
    lib/ModelFormat/Quantization.cpp:25-55), compiled from its sources into
    oracle/_ref and recorded in tests/golden/reference_pins.json;
  * the known-answer cases of tests/FlashAttentionTest.mm (LCG inputs and the
    dense fp64 causal GQA), recomputed independently in
    tests/golden/gqa_kat.npz;
  * the cost-model pins of tests/GraphIRTest.cpp:74-104 and
    tests/ConverterTest.py:170-187;
  * for DeltaNet, the transformers functions the reference's parity test
    compares against (tests/golden/delta_xcheck.npz, a cross-check: the
    reference pins another transformers version).
"""
import json
from pathlib import Path

import numpy as np
import pytest

import _inputs
import _oracle

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def pins():
    return json.loads((GOLDEN / "reference_pins.json").read_text())


def test_f32_to_f16_matches_reference_floatToHalf(pins):
    values = np.array(pins["float_to_half"]["values"], np.float32)
    expected = np.array(pins["float_to_half"]["bits"], np.uint16)
    got = _oracle.f32_to_f16_bits(values)
    np.testing.assert_array_equal(got, expected)


def test_f16_to_f32_matches_reference_halfToFloat(pins):
    bits = np.array(pins["half_to_float"]["bits"], np.uint16)
    expected = np.array(pins["half_to_float"]["values"], np.float32)
    got = _oracle.f16_bits_to_f32(bits)
    finite = np.isfinite(expected)
    np.testing.assert_array_equal(got[finite], expected[finite])
    np.testing.assert_array_equal(np.isinf(got), np.isinf(expected))


def test_f16_conversion_matches_numpy_round_to_nearest_even():
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(200000) * 10.0 ** rng.integers(-9, 6, 200000)).astype(np.float32)
    np.testing.assert_array_equal(_oracle.f32_to_f16_bits(x), x.astype(np.float16).view(np.uint16))
    every = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    finite = (every & 0x7C00) != 0x7C00
    got = _oracle.f16_bits_to_f32(every)
    np.testing.assert_array_equal(got[finite], every.view(np.float16)[finite].astype(np.float32))


def test_lcg_fill_matches_flash_attention_test_inputs():
    kat = np.load(GOLDEN / "gqa_kat.npz")
    for case in (0, 1):
        T, Hq, Hkv, D, past = kat[f"case{case}_shape"]
        q, state = _oracle.lcg_fill(179531, T * Hq * D)
        k, state = _oracle.lcg_fill(state, (past + T) * Hkv * D)
        v, state = _oracle.lcg_fill(state, (past + T) * Hkv * D)
        np.testing.assert_array_equal(q, kat[f"case{case}_q"])
        np.testing.assert_array_equal(k, kat[f"case{case}_k"])
        np.testing.assert_array_equal(v, kat[f"case{case}_v"])


def kat_case(case):
    kat = np.load(GOLDEN / "gqa_kat.npz")
    T, Hq, Hkv, D, past = (int(x) for x in kat[f"case{case}_shape"])
    q = kat[f"case{case}_q"].view(np.float16).reshape(1, T, Hq, D)
    k = kat[f"case{case}_k"].view(np.float16).reshape(1, past + T, Hkv, D)
    v = kat[f"case{case}_v"].view(np.float16).reshape(1, past + T, Hkv, D)
    return q, k, v, past, kat[f"case{case}_expected"].reshape(1, T, Hq, D)


@pytest.mark.parametrize("case", [0, 1])
def test_dense_gqa_matches_known_answers(case):
    q, k, v, past, expected = kat_case(case)
    got = _oracle.gqa_dense(q, k, v, past)
    np.testing.assert_allclose(got, expected, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("case", [0, 1])
def test_eager_fp16_path_stays_within_reference_tolerance(case):
    # The reference's decode path rounds scores and probabilities to fp16; on
    # the KAT inputs it stays within the bar the acceptance tests use.
    q, k, v, past, expected = kat_case(case)
    got = _oracle.gqa_eager_f16(q, k, v, past)
    max_abs, rel = _inputs.errors(got, expected)
    assert max_abs <= _inputs.MAX_ABS and rel <= 5e-3, (max_abs, rel)


def test_dense_gqa_batch_and_threads_are_consistent():
    q, k, v = _inputs.gqa_case(3, 5, 11, 8, 2, 16, capacity=20)
    one = _oracle.gqa_dense(q, k, v, 11, threads=1)
    many = _oracle.gqa_dense(q, k, v, 11, threads=0)
    np.testing.assert_array_equal(one, many)
    for b in range(3):
        single = _oracle.gqa_dense(q[b:b + 1], k[b:b + 1], v[b:b + 1], 11)
        np.testing.assert_array_equal(single, one[b:b + 1])


def test_dense_gqa_rows_equal_the_full_check():
    # The sampled-rows form (used where the full output is too large for a
    # CPU) gives the full check's rows bit for bit.
    q, k, v = _inputs.gqa_case(2, 40, 10, 8, 2, 64, seed=3)
    full = _oracle.gqa_dense(q, k, v, 10)
    token = np.array([0, 5, 39, 20, 39])
    head = np.array([7, 0, 3, 5, 0])
    for b in range(2):
        rows = _oracle.gqa_dense_rows(q[b, token, head], k[b], v[b], 10, 40, 8, token, head)
        np.testing.assert_array_equal(rows, full[b, token, head])


def test_delta_oracle_matches_transformers_recurrent_rule():
    d = np.load(GOLDEN / "delta_xcheck.npz")
    out, state = _oracle.delta_update(d["q"], d["k"], d["v"].view(np.float16), d["beta"],
                                      d["decay"], d["state"])
    max_abs, rel = _inputs.errors(out, d["recurrent_out"])
    assert max_abs <= 2e-3 and rel <= 1e-3, (max_abs, rel)  # output is rounded to fp16
    max_abs, rel = _inputs.errors(state, d["recurrent_state"])
    assert max_abs <= 1e-5 and rel <= 1e-5, (max_abs, rel)


def test_delta_oracle_is_chunk_partition_invariant():
    # Running T tokens at once or in two steps gives the same state and
    # outputs (the reference's partition-invariance check,
    # tests/MetalReferenceTest.py:289-296).
    c = _inputs.delta_case(2, 9, 1, 8, 2, 4, state_std=0.02, seed=5)
    full_out, full_state = _oracle.delta_update(c["q"], c["k"], c["v"], c["beta"], c["decay"],
                                                c["state"])
    cut = 4
    part = {n: a[:, :cut] for n, a in c.items() if n != "state"}
    rest = {n: a[:, cut:] for n, a in c.items() if n != "state"}
    o1, s1 = _oracle.delta_update(part["q"], part["k"], part["v"], part["beta"], part["decay"],
                                  c["state"])
    o2, s2 = _oracle.delta_update(rest["q"], rest["k"], rest["v"], rest["beta"], rest["decay"], s1)
    np.testing.assert_array_equal(np.concatenate([o1, o2], axis=1), full_out)
    np.testing.assert_array_equal(s2, full_state)


def test_cost_model_pins():
    lib = _oracle.lib()
    # tests/GraphIRTest.cpp:74-104: T=3, P=2, two query heads, head_dim 8.
    assert lib.oracle_gqa_fp_macs(3, 2, 2, 8) == 384
    # tests/ConverterTest.py:186: T=3, two value heads of 4 x 4.
    assert lib.oracle_delta_fp_macs(3, 2, 4, 4) == 288
    assert lib.oracle_gqa_pairs(128, 0) == 8256


def test_cost_model_matches_reference_records(pins):
    # The oracle's cost formulas (used to price the CPU baseline) against the
    # records of the reference's own GraphIR cost model compiled from source.
    fields = pins["attention_costs"]["fields"]
    checked = 0
    for case in pins["attention_costs"]["cases"]:
        if case["status"] != 0:
            continue
        tokens, past, _ = case["step"]
        hq, hkv, d, hk, dk, hv, dv = case["shape"]
        want = dict(zip(fields, case["record"]))
        assert _oracle.kv_append_bytes(tokens, hkv, d)[1] == want["kv_write_bytes"]
        assert _oracle.gqa_bytes(tokens, past, hq, hkv, d) == (want["gqa_read_bytes"],
                                                                want["gqa_write_bytes"])
        assert _oracle.lib().oracle_gqa_fp_macs(tokens, past, hq, d) == want["gqa_fp_macs"]
        assert _oracle.delta_bytes(tokens, hk, dk, hv, dv) == (want["delta_read_bytes"],
                                                                want["delta_write_bytes"])
        assert _oracle.lib().oracle_delta_fp_macs(tokens, hv, dk, dv) == want["delta_fp_macs"]
        checked += 1
    assert checked >= 20
