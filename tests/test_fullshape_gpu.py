"""Parity at the benchmarked shapes (3, 4 and 5), through
the C ABI, against the CPU oracle on sampled rows.

The product runs the whole configuration (every (batch, head), every query
block, the persistent / heaviest-first schedules and the long causal paths
that only these sizes reach); the oracle recomputes a row sample of every
(batch, head) -- rows spread over the sequence, always including the first
and the last row -- which it finishes in seconds.

Tolerances as for the smaller parity tests: bf16 and INT8 outputs within
2e-2 max-abs of the fp32 oracle fed the same rounded inputs, LSE within 1e-3;
INT8 logits bit-exact; the GPT-2 layer within 2e-2 * max(1, |ref|).
"""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


def _rows(n, count, seed):
    """`count` sorted query rows over [0, n): the first, the last, the last
    full tile's edges and a seeded spread."""
    rng = np.random.default_rng(seed)
    fixed = [0, 1, 127, 128, n // 2, n - 129, n - 128, n - 2, n - 1]
    extra = rng.choice(n, size=max(0, count - len(fixed)), replace=False)
    return np.unique(np.clip(np.concatenate([fixed, extra]), 0, n - 1)).astype(np.int64)


def _bf16(shape, seed, device="cuda"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(*shape, generator=g).to(torch.bfloat16).to(device)


def _check_sampled(ora, q, k, v, o, lse, causal, rows_per_head, seed):
    B, H, N, D = q.shape
    worst, worst_l = 0.0, 0.0
    scale = 1.0 / math.sqrt(D)
    for b in range(B):
        for h in range(H):
            rows = _rows(N, rows_per_head, seed + b * H + h)
            qh = q[b, h].float().cpu().numpy()[None, None]
            kh = k[b, h].float().cpu().numpy()[None, None]
            vh = v[b, h].float().cpu().numpy()[None, None]
            ref, rl = ora.attention_batched(qh, kh, vh, scale, causal, rows=rows, want_lse=True)
            got = o[b, h].float().cpu().numpy()[rows]
            worst = max(worst, float(np.abs(got - ref[0, 0, rows]).max()))
            worst_l = max(worst_l, float(np.abs(lse[b, h].cpu().numpy()[rows] - rl[0, 0, rows]).max()))
    return worst, worst_l


@pytest.mark.parametrize("causal", [True, False])
def test_config2_full_shape(gae, ora, causal):
    """Config 2: B=4, H=16, N=8192, head_dim 128, bf16, both masks; 48 rows
    of each of the 64 (batch, head) slices."""
    B, H, N, D = 4, 16, 8192, 128
    q, k, v = (_bf16((B, H, N, D), 1000 + i) for i in range(3))
    o, lse = gae.attention(q, k, v, causal=causal, return_lse=True)
    torch.cuda.synchronize()
    gae.device_status()
    err, lerr = _check_sampled(ora, q, k, v, o, lse, causal, 48, 7)
    assert err <= BF16_TOL, err
    assert lerr <= 1e-3, lerr


def test_config5_long_full_shape(gae, ora):
    """Config 5 on one GPU: one sequence of N=131072, H=8, head_dim 128,
    causal; 24 rows of each head (the oracle walks up to 131072 keys a row)."""
    B, H, N, D = 1, 8, 131072, 128
    q, k, v = (_bf16((B, H, N, D), 2000 + i) for i in range(3))
    o, lse = gae.attention(q, k, v, causal=True, return_lse=True)
    torch.cuda.synchronize()
    gae.device_status()
    err, lerr = _check_sampled(ora, q, k, v, o, lse, True, 24, 11)
    assert err <= BF16_TOL, err
    assert lerr <= 1e-3, lerr


def test_config4_attention_d64_full_shape(gae, ora):
    """The attention of config 4 alone: B=8, H=12, N=2048, head_dim 64 (the
    persistent schedule and the tensor-core row sums), causal."""
    B, H, N, D = 8, 12, 2048, 64
    q, k, v = (_bf16((B, H, N, D), 3000 + i) for i in range(3))
    o, lse = gae.attention(q, k, v, causal=True, return_lse=True)
    torch.cuda.synchronize()
    gae.device_status()
    err, lerr = _check_sampled(ora, q, k, v, o, lse, True, 32, 13)
    assert err <= BF16_TOL, err
    assert lerr <= 1e-3, lerr


def test_config3_int8_full_shape(gae, ora):
    """Config 3: B=1, H=32, N=16384, head_dim 128, non-causal, per-row int8
    Q/K; 16 rows of each head against the oracle's int8 path."""
    BH, N, D = 32, 16384, 128
    g = torch.Generator(device="cpu").manual_seed(4000)
    xq = torch.randn(BH, N, D, generator=g).cuda()
    xk = torch.randn(BH, N, D, generator=g).cuda()
    v = torch.randn(BH, N, D, generator=g).to(torch.bfloat16).cuda()
    q, sq = gae.quantize_rows_int8(xq)
    k, sk = gae.quantize_rows_int8(xk)
    o = gae.attention_int8(q, k, sq, sk, v, causal=False)
    torch.cuda.synchronize()
    gae.device_status()
    worst = 0.0
    for h in range(BH):
        rows = _rows(N, 16, 17 + h)
        ref = ora.attention_int8(q[h:h + 1].cpu().numpy(), k[h:h + 1].cpu().numpy(),
                                 sq[h:h + 1].cpu().numpy(), sk[h:h + 1].cpu().numpy(),
                                 v[h:h + 1].float().cpu().numpy(), 1 / math.sqrt(D), causal=False,
                                 rows=rows)
        worst = max(worst, float(np.abs(o[h].float().cpu().numpy()[rows] - ref[0, rows]).max()))
    assert worst <= BF16_TOL, worst


@pytest.mark.parametrize("causal", [False, True])
def test_int8_attention_kernel_logits_bit_exact(gae, ora, causal):
    """The int32 QK^T of the INT8 attention kernel itself (not a sibling
    kernel): the same launch that produces O writes the logits it read from
    TMEM; they equal the oracle's dot_int8 bit for bit, and O equals the
    plain call's O bit for bit."""
    BH, N, D = 2, 2048 + 76, 128
    g = torch.Generator(device="cpu").manual_seed(4100)
    q, sq = gae.quantize_rows_int8(torch.randn(BH, N, D, generator=g).cuda())
    k, sk = gae.quantize_rows_int8(torch.randn(BH, N, D, generator=g).cuda())
    v = torch.randn(BH, N, D, generator=g).to(torch.bfloat16).cuda()
    logits = torch.full((BH, N, N), -1, dtype=torch.int32, device="cuda")
    o_dump = gae.attention_int8(q, k, sq, sk, v, causal=causal, logits_out=logits)
    o = gae.attention_int8(q, k, sq, sk, v, causal=causal)
    torch.cuda.synchronize()
    gae.device_status()
    ref = ora.int8_logits(q.cpu().numpy(), k.cpu().numpy())
    got = logits.cpu().numpy()
    if causal:  # only the visible (and diagonal-tile) entries are computed
        mask = np.tril(np.ones((N, N), bool))[None].repeat(BH, 0)
        assert np.array_equal(got[mask], ref[mask])
    else:
        assert np.array_equal(got, ref)
    assert torch.equal(o_dump, o)


def test_config4_gpt2_layer_full_shape(gae, ora):
    """One GPT-2-small layer of config 4 at its full shape (B=8, S=2048,
    d_model 768, 12 heads, MLP 3072); sequences 0 and 7 recomputed by the
    oracle (a sequence is independent of the others)."""
    B, S, Dm, H, F = 8, 2048, 768, 12, 3072
    layer = gae.Gpt2Layer.random(Dm, H, F, device="cuda", seed=5)
    x = _bf16((B, S, Dm), 5000)
    y = layer.forward(x)
    torch.cuda.synchronize()
    gae.device_status()
    w = {k_: v_.float().cpu().numpy() for k_, v_ in layer.w.items()}
    for k_ in ("w_qkv", "w_proj", "w_fc", "w_fc2"):
        w[k_] = np.ascontiguousarray(w[k_].T)  # the oracle takes [in, out]
    w = dict(ln1_g=w["ln1_gamma"], ln1_b=w["ln1_beta"], wqkv=w["w_qkv"], bqkv=w["b_qkv"],
             wproj=w["w_proj"], bproj=w["b_proj"], ln2_g=w["ln2_gamma"], ln2_b=w["ln2_beta"],
             wfc=w["w_fc"], bfc=w["b_fc"], wfc2=w["w_fc2"], bfc2=w["b_fc2"])
    worst = 0.0
    for b in (0, B - 1):
        ref = ora.gpt2_layer(x[b].float().cpu().numpy(), 1, S, Dm, H, F, 1e-5, w, round_bf16=True)
        got = y[b].float().cpu().numpy()
        worst = max(worst, float((np.abs(got - ref) / np.maximum(1.0, np.abs(ref))).max()))
    assert worst <= 2e-2, worst
