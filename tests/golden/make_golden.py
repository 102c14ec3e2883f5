"""Generates the committed golden fixtures under tests/golden/.

Run from the repository root in a container that has the reference tree and
transformers installed:  python tests/golden/make_golden.py <reference tree>

Fixtures (all small):
  gqa_kat.npz        The two known-answer cases of the reference's
                     tests/FlashAttentionTest.mm:107-108 (GqaParams {19,4,2,12,0}
                     and {7,4,2,256,33}): the LCG input bits of :28-36 and the
                     fp64 dense causal GQA outputs, computed here with numpy
                     (an implementation independent of oracle/oracle.c).
  delta_xcheck.npz   A small Gated-DeltaNet case and its outputs/final state from
                     transformers' torch_recurrent_gated_delta_rule and
                     torch_chunk_gated_delta_rule (models/qwen3_5), run in fp64.
                     The reference's own parity test compares its DeltaNet
                     against these functions (tests/MetalReferenceTest.py); it
                     pins transformers 5.20.2, this fixture was made with the
                     installed version recorded in the file.
  reference_pins.json  Values computed by the reference's own C++ compiled from
                     its sources (oracle/_ref/libllmi_ref.so, built by
                     `make -C oracle ref REFERENCE=<tree>`): floatToHalf /
                     halfToFloat on edge-case values, and the GraphIR effects
                     and cost of KvAppend / CausalGqa / DeltaUpdate over a grid
                     of step shapes.
"""
from __future__ import annotations

import ctypes
import json
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(HERE.parent))

import _inputs  # noqa: E402
import _oracle  # noqa: E402

KAT_SHAPES = [(19, 4, 2, 12, 0), (7, 4, 2, 256, 33)]  # tokens, Hq, Hkv, D, past


def lcg_bits(state: int, n: int) -> tuple[np.ndarray, int]:
    """Pure-Python restatement of the LCG fill (independent of oracle.c)."""
    vals = np.empty(n, np.float32)
    for i in range(n):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        vals[i] = np.float32((state >> 24) - 128) / np.float32(64.0)
    return vals.astype(np.float16).view(np.uint16), state


def dense_gqa_numpy(q, k, v, past):
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    g = Hq // Hkv
    out = np.zeros((T, Hq, D), np.float64)
    for t in range(T):
        vis = past + t + 1
        for h in range(Hq):
            kk = k[:vis, h // g].astype(np.float64)
            vv = v[:vis, h // g].astype(np.float64)
            s = kk @ q[t, h].astype(np.float64) / np.sqrt(D)
            w = np.exp(s - s.max())
            out[t, h] = (w @ vv) / w.sum()
    return out


def make_gqa_kat():
    arrays = {}
    for i, (T, Hq, Hkv, D, past) in enumerate(KAT_SHAPES):
        state = 179531
        qb, state = lcg_bits(state, T * Hq * D)
        kb, state = lcg_bits(state, (past + T) * Hkv * D)
        vb, state = lcg_bits(state, (past + T) * Hkv * D)
        q = qb.view(np.float16).reshape(T, Hq, D)
        k = kb.view(np.float16).reshape(past + T, Hkv, D)
        v = vb.view(np.float16).reshape(past + T, Hkv, D)
        arrays[f"case{i}_shape"] = np.array([T, Hq, Hkv, D, past], np.int64)
        arrays[f"case{i}_q"] = qb
        arrays[f"case{i}_k"] = kb
        arrays[f"case{i}_v"] = vb
        arrays[f"case{i}_expected"] = dense_gqa_numpy(q, k, v, past)
    np.savez_compressed(HERE / "gqa_kat.npz", **arrays)


def make_delta_xcheck():
    import torch
    import transformers
    from transformers.models.qwen3_5 import modeling_qwen3_5 as m

    B, T, Hk, dk, Hv, dv = 2, 70, 2, 16, 4, 8
    case = _inputs.delta_case(B, T, Hk, dk, Hv, dv, state_std=0.02, seed=4242)
    ratio = Hv // Hk
    to = lambda a: torch.from_numpy(np.asarray(a, np.float64))
    # transformers scales q by 1/sqrt(dk) itself: undo the builder's scale.
    q = to(case["q"]).reshape(B, T, Hk, dk) * np.sqrt(dk)
    k = to(case["k"]).reshape(B, T, Hk, dk)
    q = q.repeat_interleave(ratio, dim=2)
    k = k.repeat_interleave(ratio, dim=2)
    v = to(case["v"].astype(np.float32)).reshape(B, T, Hv, dv)
    g = torch.log(to(case["decay"]))
    beta = to(case["beta"])
    s0 = to(case["state"])
    out_r, state_r = m.torch_recurrent_gated_delta_rule(q, k, v, g, beta, s0.clone(), True)
    out_c, state_c = m.torch_chunk_gated_delta_rule(q, k, v, g, beta, 64, s0.clone(), True)
    arrays = {k2: np.asarray(v2) for k2, v2 in case.items()}
    arrays["v"] = case["v"].view(np.uint16)
    arrays.update(
        shape=np.array([B, T, Hk, dk, Hv, dv], np.int64),
        recurrent_out=out_r.reshape(B, T, Hv * dv).numpy(),
        recurrent_state=state_r.numpy(),
        chunk_out=out_c.reshape(B, T, Hv * dv).numpy(),
        chunk_state=state_c.numpy(),
        transformers_version=np.array(transformers.__version__),
    )
    np.savez_compressed(HERE / "delta_xcheck.npz", **arrays)


def make_reference_pins(reference: Path):
    subprocess.run(["make", "-C", str(ROOT / "oracle"), "ref", f"REFERENCE={reference}"],
                   check=True, capture_output=True)
    ref = _oracle.reference_shim()
    assert ref is not None
    specials = [0.0, -0.0, 1.0, -2.5, 65504.0, 65519.99, 65520.0, 1e6, -1e6, 6.1035156e-05,
                6.0975552e-05, 5.9604645e-08, 2.9802322e-08, 2.9802326e-08, 1e-9, 1.0009765625,
                1.00048828125, 1.00146484375, 0.333333, float("inf"), float("-inf")]
    rng = np.random.default_rng(7)
    randoms = np.concatenate([rng.standard_normal(200) * 10.0 ** rng.integers(-9, 5, 200),
                              rng.standard_normal(56)]).astype(np.float32).tolist()
    values = [float(np.float32(x)) for x in specials + randoms]
    half = [int(ref.ref_float_to_half(x)) for x in values]
    bits = list(range(0, 65536, 97)) + [0x7c00, 0xfc00, 0x0001, 0x03ff, 0x0400, 0x7bff]
    back = [float(ref.ref_half_to_float(b)) for b in bits]

    n = ref.ref_field_count()
    records = []
    for tokens, past, capacity in [(3, 2, 8), (1, 0, 1), (1, 4096, 8192), (128, 0, 128),
                                   (7, 33, 40), (19, 0, 19), (4096, 0, 4096), (64, 64, 200)]:
        for shape in [(2, 1, 8, 1, 4, 2, 4), (16, 4, 256, 16, 128, 32, 128), (4, 2, 12, 2, 7, 4, 5)]:
            rec = (ctypes.c_uint64 * n)()
            status = ref.ref_attention_costs(tokens, past, capacity, *shape, rec)
            records.append(dict(step=[tokens, past, capacity], shape=list(shape),
                                status=status, record=list(rec)))
    pins = dict(float_to_half=dict(values=values, bits=half),
                half_to_float=dict(bits=bits, values=back),
                attention_costs=dict(
                    fields=["kv_write_bytes", "kv_begin", "kv_length", "kv_version_before",
                            "kv_version_after", "gqa_read_bytes", "gqa_write_bytes",
                            "gqa_fp_macs", "gqa_begin", "gqa_length", "gqa_version_before",
                            "gqa_version_after", "delta_read_bytes", "delta_write_bytes",
                            "delta_fp_macs"],
                    shape_fields=["queryHeads", "kvHeads", "headDim", "keyHeads", "keyDim",
                                  "valueHeads", "valueDim"],
                    cases=records))
    (HERE / "reference_pins.json").write_text(json.dumps(pins, indent=1) + "\n")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    make_gqa_kat()
    make_delta_xcheck()
    make_reference_pins(Path(sys.argv[1]))
    print("fixtures written to", HERE)
