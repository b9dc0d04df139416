"""gae_layer_fwd_static: the layer forward for callers that cannot allocate
device memory (allocator callbacks, plugins whose host owns all device
allocations, real-time paths).  Called through the C ABI, it must give the
same output as gae_layer_fwd with a caller workspace, on two calls in a row
(the shared static workspace keeps the previous call's contents), within the
layer tolerance of tests/test_layer_gpu.py: |a - b| <= 2e-2 * max(1, |b|).
This file is collected last so that a run stopping at the first failure has
already run every other test; it also passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _within(a, b):
    return float((np.abs(a - b) / np.maximum(1.0, np.abs(b))).max())


def _static_call(gae, layer, x, out):
    B, S, D = x.shape
    args = gae.LayerArgs(x.data_ptr(), out.data_ptr(), B, S, D, layer.heads, layer.d_ff,
                         layer.eps, None, 0)
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return gae.lib().gae_layer_fwd_static(C.byref(args), C.byref(layer._cw), st)


def test_static_workspace_layer_matches_allocating_entry(gae):
    D, H, F = 768, 12, 3072
    layer = gae.Gpt2Layer.random(D, H, F, seed=31)
    for call, (B, S) in enumerate([(1, 256), (2, 384)]):
        g = torch.Generator().manual_seed(40 + call)
        x = torch.randn(B, S, D, generator=g).bfloat16().cuda()
        ref = layer.forward(x)
        out = torch.full_like(x, float("nan"))
        assert _static_call(gae, layer, x, out) == 0
        torch.cuda.synchronize()
        gae.device_status()
        assert _within(out.float().cpu().numpy(), ref.float().cpu().numpy()) <= 2e-2


def test_static_workspace_rejects_oversized_shape(gae):
    layer = gae.Gpt2Layer.random(768, 12, 3072, seed=32)
    x = torch.zeros(8, 2048, 768, dtype=torch.bfloat16, device="cuda")
    assert _static_call(gae, layer, x, torch.empty_like(x)) == 2  # GAE_ERR_UNSUPPORTED
    buf = C.create_string_buffer(512)
    gae.lib().gae_last_error(buf, 512)
    assert b"static workspace" in buf.value
