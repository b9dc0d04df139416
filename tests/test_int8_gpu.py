"""INT8 path through the C ABI against the oracle.

Bar: the int32 QK^T logits are bit-exact (tcgen05 kind::i8 vs the reference's
dot_int8 restated in the oracle); the attention output is within 2e-2
max-abs of the oracle fed the same int8 inputs, fp32 scales and bf16 V.
"""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _i8(shape, seed, lo=-127, hi=127):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, shape, generator=g, dtype=torch.int16).to(torch.int8)


@pytest.mark.parametrize("BH,Nq,Nkv", [(1, 128, 128), (2, 300, 257), (3, 1024, 640)])
def test_int8_logits_bit_exact(gae, ora, BH, Nq, Nkv):
    q = _i8((BH, Nq, 128), 1)
    k = _i8((BH, Nkv, 128), 2)
    got = gae.int8_logits(q.cuda(), k.cuda())
    ref = ora.int8_logits(q.numpy(), k.numpy())
    assert np.array_equal(got.cpu().numpy(), ref)


def test_int8_logits_extreme_values(gae, ora):
    # -128 * -128 * 128 = 2^21: int32 accumulation must stay exact.
    q = torch.full((1, 128, 128), -128, dtype=torch.int8)
    k = torch.full((1, 128, 128), -128, dtype=torch.int8)
    k[0, 5] = 127
    got = gae.int8_logits(q.cuda(), k.cuda()).cpu().numpy()
    assert np.array_equal(got, ora.int8_logits(q.numpy(), k.numpy()))
    assert got[0, 0, 0] == 128 * 128 * 128


def _int8_case(gae, ora, BH, N, causal, seed=0, zero_rows=()):
    g = torch.Generator().manual_seed(seed)
    xq = torch.randn(BH, N, 128, generator=g)
    xk = torch.randn(BH, N, 128, generator=g)
    for r in zero_rows:
        xq[0, r] = 0
    v = torch.randn(BH, N, 128, generator=g).bfloat16()
    q, sq = gae.quantize_rows_int8(xq.cuda())
    k, sk = gae.quantize_rows_int8(xk.cuda())
    o = gae.attention_int8(q, k, sq, sk, v.cuda(), causal=causal)
    torch.cuda.synchronize()
    gae.device_status()
    ref = ora.attention_int8(q.cpu().numpy(), k.cpu().numpy(), sq.cpu().numpy(),
                             sk.cpu().numpy(), v.float().numpy(), 1 / math.sqrt(128),
                             causal=causal)
    err = float(np.abs(o.float().cpu().numpy() - ref).max())
    assert err <= 2e-2, err


@pytest.mark.parametrize("causal", [False, True])
def test_int8_attention(gae, ora, causal):
    _int8_case(gae, ora, 2, 512, causal)


@pytest.mark.parametrize("N", [4, 132, 1000])
def test_int8_attention_ragged(gae, ora, N):
    _int8_case(gae, ora, 1, N, False, seed=N)
    _int8_case(gae, ora, 1, N, True, seed=N + 1)


def test_int8_attention_zero_query_rows(gae, ora):
    _int8_case(gae, ora, 1, 256, False, zero_rows=(0, 7, 200))
    _int8_case(gae, ora, 1, 256, True, zero_rows=(0, 7, 200))


def test_int8_rejects_bad_shapes(gae):
    q = torch.zeros(1, 128, 64, dtype=torch.int8, device="cuda")
    s = torch.ones(1, 128, device="cuda")
    v = torch.zeros(1, 128, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(gae.GAEError):
        gae.attention_int8(q, q, s, s, v)


def test_reference_int8_kernel_pins_oracle_and_product(gae, ora):
    """The reference's own INT8 Waller kernel (cuda_src/waller_operator_int8.cu:
    27-68, built from its source into oracle/_ref: causal, one global
    qk_scale, V int8 / v_scale) against the oracle's INT8 restatement (unit row
    scales, the same scale, V = v / v_scale in fp32: max-abs <= 1e-5 of the
    largest output) and this library's INT8 attention (V rounded to bf16,
    output bf16: 2e-2 max-abs)."""
    L = ora.ref_waller_int8()
    if L is None:
        pytest.skip("reference INT8 kernel not built (no reference tree where build() ran)")
    rng = np.random.default_rng(31)
    n, d = 1000, 128
    q, k, v = (rng.integers(-127, 128, (n, d)).astype(np.int8) for _ in range(3))
    qk_scale, v_scale = 1.0 / (math.sqrt(d) * 127.0 * 8.0), 127.0
    dev = [torch.from_numpy(a).cuda() for a in (q, k, v)]
    od = torch.empty(n, d, dtype=torch.float32, device="cuda")
    assert L.ref_waller_int8_fwd(dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), od.data_ptr(), n, d,
                                 qk_scale, v_scale, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    ref_gpu = od.cpu().numpy()
    ones = np.ones((1, n), np.float32)
    vf = (v.astype(np.float32) / np.float32(v_scale))
    ora_out = ora.attention_int8(q[None], k[None], ones, ones, vf[None], qk_scale, causal=True)[0]
    assert float(np.abs(ora_out - ref_gpu).max()) <= 1e-5 * float(np.abs(ref_gpu).max())
    got = gae.attention_int8(dev[0][None].contiguous(), dev[1][None].contiguous(),
                             torch.ones(1, n, device="cuda"), torch.ones(1, n, device="cuda"),
                             torch.from_numpy(vf[None]).cuda().bfloat16(), causal=True, scale=qk_scale)
    assert float(np.abs(got.float().cpu().numpy()[0] - ref_gpu).max()) <= 2e-2
