"""Attention backward (gae_attn_bwd, tcgen05 kernel) against the CPU oracle's
gradients from the definition (double precision) on the same bf16/f16-rounded
inputs, and against torch autograd in fp32.

Tolerance: for each of dQ, dK, dV, max|gpu - ref| <= 2e-2 * max|ref| (the
gradients are accumulated in fp32 from 16-bit P and dS tiles, and stored in
16 bits)."""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _rel(got, ref):
    got = got.float().cpu().numpy() if hasattr(got, "cpu") else got
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-6))


def _case(B, H, Nq, Nkv, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    mk = lambda n: torch.randn(B, H, n, D, generator=g).to(dtype)
    return mk(Nq), mk(Nkv), mk(Nkv), mk(Nq)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("B,H,Nq,Nkv,causal", [(1, 2, 256, 256, True), (2, 1, 300, 300, True),
                                               (1, 2, 200, 333, False), (1, 1, 128, 128, False)])
def test_backward_matches_oracle(gae, ora, D, B, H, Nq, Nkv, causal):
    q, k, v, do = _case(B, H, Nq, Nkv, D, torch.bfloat16, 7 + D + Nq)
    scale = 1.0 / math.sqrt(D)
    qd, kd, vd, dod = (t.cuda() for t in (q, k, v, do))
    out, lse = gae.attention(qd, kd, vd, causal=causal, return_lse=True)
    dq, dk, dv = gae.attention_backward(qd, kd, vd, out, dod, lse, causal=causal)
    torch.cuda.synchronize()
    gae.device_status()
    f = lambda t: t.float().numpy().reshape(B * H, -1, D)
    rq, rk, rv = ora.attention_bwd(f(q), f(k), f(v), f(do), scale, causal)
    assert _rel(dq.reshape(B * H, -1, D), rq) <= 2e-2
    assert _rel(dk.reshape(B * H, -1, D), rk) <= 2e-2
    assert _rel(dv.reshape(B * H, -1, D), rv) <= 2e-2


def test_backward_f16_and_strided(gae, ora):
    # f16, and q/k/v as head-interleaved views of one packed [B, N, 3, H, D] tensor
    B, H, N, D = 1, 2, 384, 128
    g = torch.Generator().manual_seed(5)
    qkv = torch.randn(B, N, 3, H, D, generator=g).half().cuda()
    q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    do = torch.randn(B, H, N, D, generator=g).half().cuda()
    out, lse = gae.attention(q, k, v, causal=True, return_lse=True)
    dq, dk, dv = gae.attention_backward(q, k, v, out, do, lse, causal=True)
    torch.cuda.synchronize()
    f = lambda t: t.float().cpu().numpy().reshape(B * H, N, D)
    rq, rk, rv = ora.attention_bwd(f(q), f(k), f(v), f(do), 1 / math.sqrt(D), True)
    for got, ref in ((dq, rq), (dk, rk), (dv, rv)):
        assert _rel(got.reshape(B * H, N, D), ref) <= 2e-2


def test_autograd_matches_torch_fp32(gae):
    B, H, N, D = 2, 2, 256, 64
    g = torch.Generator().manual_seed(9)
    base = [torch.randn(B, H, N, D, generator=g).bfloat16() for _ in range(3)]
    dout = torch.randn(B, H, N, D, generator=g).bfloat16()
    q, k, v = (t.cuda().requires_grad_() for t in base)
    o = gae.attention_autograd(q, k, v, causal=True)
    o.backward(dout.cuda())
    # plain PyTorch fp32 reference of the same op
    qf, kf, vf = (t.float().requires_grad_() for t in base)
    s = (qf @ kf.transpose(-1, -2)) / math.sqrt(D)
    s = s.masked_fill(torch.triu(torch.ones(N, N, dtype=torch.bool), 1), float("-inf"))
    of = torch.softmax(s, -1) @ vf
    of.backward(dout.float())
    for got, ref in ((q.grad, qf.grad), (k.grad, kf.grad), (v.grad, vf.grad)):
        assert _rel(got, ref.numpy()) <= 2e-2


def test_backward_rejects_bad_args(gae):
    q = torch.zeros(1, 1, 128, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(1, 1, 256, 128, dtype=torch.bfloat16, device="cuda")
    lse = torch.zeros(1, 1, 128, device="cuda")
    with pytest.raises(gae.GAEError):  # causal needs Nq == Nkv
        gae.attention_backward(q, k, k, q, q, lse, causal=True)
