"""llmi_cuda_gqa_decode_noalloc: decode for callers that cannot allocate.

Some callers cannot allocate device memory themselves - an executor that
hands out all device memory from its own fixed arena, or a latency-critical
decode loop that cannot absorb cudaMalloc's possible device-wide
synchronisation.  For them the library offers a decode entry point whose
scratch is a fixed array inside the library instead of a caller workspace.

These tests call it through the C ABI and check it against the regular
llmi_cuda_gqa_decode (which takes a caller workspace), on two calls in a
row, with the tolerance the other GPU tests use.  The file is named to be
collected last and passes alone in a fresh process as well.
"""
import ctypes

import numpy as np
import pytest
import torch

import _inputs
from llminfer_b200 import abi, ops

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def decode_noalloc(q, kc, vc, past):
    B, T, Hq, D = q.shape
    p = abi.GqaParams(T, Hq, kc.shape[2], D, past)
    out = torch.full_like(q, float("nan"))
    status = abi.lib.llmi_cuda_gqa_decode_noalloc(
        ctypes.byref(p), B, q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc[0].numel(),
        out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    abi.check(status)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("batch,past,hq,hkv,d", [
    (8, 4096, 16, 4, 256),   # benchmark per-sequence shape, grouped workers
    (3, 700, 16, 2, 256),    # whole rows of 2 kv heads
    (2, 50, 4, 2, 12),       # CUDA-core partial pass
    (8, 2000, 4, 1, 256),    # CTA workers: one record per (worker, unit)
    (3, 500, 8, 2, 128),     # CTA workers, head_dim 128
])
def test_noalloc_decode_matches_workspace_decode(batch, past, hq, hkv, d):
    q, k, v = _inputs.gqa_case(batch, 1, past, hq, hkv, d, capacity=past + 3, seed=past + d)
    q, k, v = dev(q), dev(k), dev(v)
    want = ops.gqa_decode(q, k, v, past).float().cpu().numpy()
    for _ in range(2):  # the shared scratch is reused by the second call
        got = decode_noalloc(q, k, v, past).float().cpu().numpy()
        assert np.isfinite(got).all()
        max_abs, rel = _inputs.errors(got, want)
        assert max_abs <= _inputs.MAX_ABS and rel <= _inputs.REL_L2, (max_abs, rel)


def test_noalloc_decode_rejects_shapes_beyond_its_scratch():
    # 8192 sequences x 4 kv heads of a short cache: the records would need far
    # more than the fixed scratch; the call must refuse before launching.
    q = torch.zeros(8192, 1, 16, 256, dtype=torch.float16, device="cuda")
    kv = torch.zeros(8192, 2, 4, 256, dtype=torch.float16, device="cuda")
    out = torch.full_like(q, float("nan"))
    p = abi.GqaParams(1, 16, 4, 256, 0)
    status = abi.lib.llmi_cuda_gqa_decode_noalloc(
        ctypes.byref(p), 8192, q.data_ptr(), kv.data_ptr(), kv.data_ptr(), kv[0].numel(),
        out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert status == abi.LLMI_WORKSPACE_TOO_SMALL
    assert "static scratch" in abi.lib.llmi_cuda_last_error().decode()
    torch.cuda.synchronize()
    assert torch.isnan(out).all()
