"""Failure detection on the GPU without a GPU fault: a bounded device-side wait
that runs out sets the error word, the host turns it into LLMI_DEVICE_TIMEOUT,
and a session whose step failed after launch is invalid until reset - the
reference's rule (MetalExecutor.mm:259-260, 285-298).  The wait that runs out
is the library's self-test kernel (an mbarrier nothing completes, 1 ms bound);
the context stays usable afterwards.
"""
import pytest
import torch

from llminfer_b200 import abi, ops

pytestmark = pytest.mark.gpu

KINDS = [abi.LAYER_DELTANET, abi.LAYER_GQA]
SHAPE = dict(query_heads=8, kv_heads=2, head_dim=256, key_heads=2, key_dim=128,
             value_heads=4, value_dim=128)


def test_timed_out_wait_reports_device_timeout_and_clears():
    ops.poll_error()  # clean start
    ops.selftest_wait_timeout(1000)
    with pytest.raises(abi.LlmiError) as err:
        ops.poll_error()
    assert err.value.status == abi.LLMI_DEVICE_TIMEOUT
    ops.poll_error()  # the word was read and cleared
    # The context still runs kernels correctly.
    q = torch.randn(1, 4, 8, 256, device="cuda").half()
    kc = torch.randn(1, 4, 2, 256, device="cuda").half()
    out = ops.gqa_prefill(q, kc, kc.clone(), 0)
    ops.poll_error()
    assert torch.isfinite(out.float()).all()


def layers(batch, tokens, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    F = torch.nn.functional
    res = []
    for kind in KINDS:
        if kind == abi.LAYER_GQA:
            q = torch.randn(batch, tokens, 8, 256, generator=g, device="cuda").half()
            k = torch.randn(batch, tokens, 2, 256, generator=g, device="cuda").half()
            v = torch.randn(batch, tokens, 2, 256, generator=g, device="cuda").half()
            res.append(ops.LayerTensors(q=q, k=k, v=v, out=torch.empty_like(q)))
        else:
            q = F.normalize(torch.randn(batch, tokens, 2, 128, generator=g, device="cuda"), dim=-1)
            k = F.normalize(torch.randn(batch, tokens, 2, 128, generator=g, device="cuda"), dim=-1)
            v = torch.randn(batch, tokens, 4 * 128, generator=g, device="cuda").half()
            beta = torch.rand(batch, tokens, 4, generator=g, device="cuda")
            decay = torch.rand(batch, tokens, 4, generator=g, device="cuda") * 0.5 + 0.5
            res.append(ops.LayerTensors(q=(q / 128 ** 0.5).reshape(batch, tokens, -1).contiguous(),
                                        k=k.reshape(batch, tokens, -1).contiguous(), v=v,
                                        out=torch.empty_like(v), beta=beta, decay=decay))
    return res


def test_failed_step_invalidates_session_until_reset():
    ops.poll_error()
    session = ops.AttentionSession(KINDS, 2, 64, **SHAPE)
    try:
        session.step(8, layers(2, 8, 1))
        assert session.past == 8 and not session.invalid
        session.inject_fault(1000)
        with pytest.raises(abi.LlmiError) as err:
            session.step(4, layers(2, 4, 2))
        assert err.value.status == abi.LLMI_DEVICE_TIMEOUT
        assert session.invalid
        assert session.past == 8  # past advances only on success
        with pytest.raises(abi.LlmiError) as err:
            session.step(1, layers(2, 1, 3))
        assert err.value.status == abi.LLMI_SESSION_INVALID
        session.reset()
        assert not session.invalid and session.past == 0
        session.step(8, layers(2, 8, 1))
        assert session.past == 8
    finally:
        session.close()
    ops.poll_error()


def test_cancelled_injection_leaves_step_untouched():
    session = ops.AttentionSession(KINDS, 1, 16, **SHAPE)
    try:
        session.inject_fault(1000)
        session.inject_fault(0)
        session.step(4, layers(1, 4, 5))
        assert session.past == 4 and not session.invalid
    finally:
        session.close()
