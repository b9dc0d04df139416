"""Failure detection on the GPU without a fault: a bounded device wait on a
barrier that nothing completes gives up after a short limit, records its site,
and the host reads GAE_ERR_TIMEOUT; the context stays usable afterwards."""
import ctypes as C

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(gae):
    gae.device_status()  # clear any earlier record
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert gae.lib().gae_debug_wait_timeout(50_000_000, stream) == 0  # 50 ms
    with pytest.raises(gae.GAEError) as err:
        gae.device_status()
    assert err.value.status == 6 and "0x901" in str(err.value)
    gae.device_status()  # the record was reset by the read
    q = torch.randn(1, 2, 256, 128, device="cuda").bfloat16()
    o = gae.attention(q, q, q, causal=True)
    torch.cuda.synchronize()
    gae.device_status()
    assert torch.isfinite(o.float()).all()


def test_wait_timeout_limit_is_checked(gae):
    assert gae.lib().gae_debug_wait_timeout(5_000_000_000, None) == 1  # above 1 s
