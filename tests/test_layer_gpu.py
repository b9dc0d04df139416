"""Fused pre-norm layer kernels (tcgen05 GEMM with fused epilogues, LayerNorm,
the whole GPT-2 layer and stack) against the CPU oracle, through the C ABI.

Tolerance (bf16 activations, fp32 accumulation): |gpu - ref| <= 2e-2 *
max(1, |ref|) elementwise, i.e. 2e-2 max-abs where |ref| <= 1 and 2e-2
relative above, which admits one bf16 rounding step of the output (2^-8
relative) and the fp32 summation-order differences.  The oracle rounds every
tensor the GPU stores between kernels to bf16 at the same points.
"""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def within(got, ref, tol=2e-2):
    err = np.abs(got - ref) / np.maximum(1.0, np.abs(ref))
    return float(err.max())


def _bf(shape, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).bfloat16()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 512, 768), (1000, 2304, 768)])
@pytest.mark.parametrize("epi", ["bias", "gelu", "residual", "none"])
def test_linear_epilogues(gae, ora, M, N, K, epi):
    x, w = _bf((M, K), 1), _bf((N, K), 2, 0.05)
    b = torch.randn(N, generator=torch.Generator().manual_seed(3))
    r = _bf((M, N), 4)
    y = gae.linear(x.cuda(), w.cuda(), bias=None if epi == "none" else b.cuda(),
                   res=r.cuda() if epi == "residual" else None, gelu=epi == "gelu")
    ref = x.float() @ w.float().T
    if epi != "none":
        ref = ref + b
    if epi == "gelu":
        ref = torch.tensor(np.vectorize(ora.gelu)(ref.numpy()), dtype=torch.float32)
    if epi == "residual":
        ref = ref + r.float()
    assert within(y.float().cpu().numpy(), ref.numpy()) <= 2e-2


def test_linear_rejects_unsupported(gae):
    x = torch.zeros(128, 100, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(256, 100, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(gae.GAEError):
        gae.linear(x, w)


def test_layernorm_rows(gae, ora):
    x = _bf((1000, 768), 5, 3.0)
    g = torch.rand(768, generator=torch.Generator().manual_seed(6)) + 0.5
    b = torch.randn(768, generator=torch.Generator().manual_seed(7))
    y = gae.layernorm_rows(x.cuda(), g.cuda(), b.cuda(), 1e-5)
    ref = ora.layernorm_batched(x.float().numpy(), g.numpy(), b.numpy(), 1000, 768, 1e-5)
    assert within(y.float().cpu().numpy(), ref.reshape(1000, 768)) <= 2e-2
    # fused residual: LN(x + r) with the rounded sum written out
    r = _bf((1000, 768), 8)
    s = torch.empty_like(x).cuda()
    y2 = gae.layernorm_rows(x.cuda(), g.cuda(), b.cuda(), 1e-5, res=r.cuda(), sum_out=s)
    ssum = (x.float() + r.float()).bfloat16()
    assert torch.equal(s.cpu(), ssum)
    ref2 = ora.layernorm_batched(ssum.float().numpy(), g.numpy(), b.numpy(), 1000, 768, 1e-5)
    assert within(y2.float().cpu().numpy(), ref2.reshape(1000, 768)) <= 2e-2


def _oracle_weights(layer):
    w = {k: v.float().cpu().numpy() for k, v in layer.w.items()}
    for k in ("w_qkv", "w_proj", "w_fc", "w_fc2"):
        w[k] = np.ascontiguousarray(w[k].T)  # oracle takes [in, out]
    return dict(ln1_g=w["ln1_gamma"], ln1_b=w["ln1_beta"], wqkv=w["w_qkv"], bqkv=w["b_qkv"],
                wproj=w["w_proj"], bproj=w["b_proj"], ln2_g=w["ln2_gamma"], ln2_b=w["ln2_beta"],
                wfc=w["w_fc"], bfc=w["b_fc"], wfc2=w["w_fc2"], bfc2=w["b_fc2"])


def _randomise_biases(layer, seed):
    g = torch.Generator().manual_seed(seed)
    for k in ("b_qkv", "b_proj", "b_fc", "b_fc2", "ln1_beta", "ln2_beta"):
        layer.w[k].copy_(torch.randn(layer.w[k].shape, generator=g) * 0.1)
    for k in ("ln1_gamma", "ln2_gamma"):
        layer.w[k].copy_(1 + 0.1 * torch.randn(layer.w[k].shape, generator=g))


@pytest.mark.parametrize("B,S", [(2, 256), (1, 300)])
def test_gpt2_layer_matches_oracle(gae, ora, B, S):
    D, H, F = 768, 12, 3072
    layer = gae.Gpt2Layer.random(D, H, F, seed=11)
    _randomise_biases(layer, 12)
    x = _bf((B, S, D), 13)
    y = layer.forward(x.cuda())
    torch.cuda.synchronize()
    gae.device_status()
    ref = ora.gpt2_layer(x.float().numpy().reshape(B * S, D), B, S, D, H, F, 1e-5,
                         _oracle_weights(layer), round_bf16=True)
    assert within(y.float().cpu().numpy().reshape(B * S, D), ref) <= 2e-2


def test_gpt2_stack_and_in_place(gae, ora):
    B, S, D, H, F = 1, 256, 768, 12, 3072
    layers = [gae.Gpt2Layer.random(D, H, F, seed=20 + i) for i in range(3)]
    x = _bf((B, S, D), 21)
    y = gae.layer_stack_forward(layers, x.cuda())
    # The stack is exactly the layers applied one after another ...
    seq = x.cuda()
    for l in layers:
        seq = l.forward(seq)
    assert torch.equal(seq.cpu(), y.cpu())
    # ... and tracks the oracle within the per-layer tolerance times the depth
    # (bf16 rounding differences compound from layer to layer).
    ref = x.float().numpy().reshape(B * S, D)
    for l in layers:
        ref = ora.gpt2_layer(ref, B, S, D, H, F, 1e-5, _oracle_weights(l), round_bf16=True)
    assert within(y.float().cpu().numpy().reshape(B * S, D), ref) <= 2e-2 * len(layers)
    # x and out may alias
    xd = x.cuda()
    gae.layer_stack_forward(layers, xd, out=xd)
    assert torch.equal(xd.cpu(), y.cpu())


def _rel(got, ref):
    """max |got - ref| / max |ref| (the fp32 tolerance of the crate drop-ins)."""
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def _crate_weights(rng, h, m):
    return dict(wq=rng.standard_normal(h * h) * 0.05, wk=rng.standard_normal(h * h) * 0.05,
                wv=rng.standard_normal(h * h) * 0.05, wo=rng.standard_normal(h * h) * 0.05,
                ln1_gamma=1 + 0.1 * rng.standard_normal(h), ln1_beta=0.1 * rng.standard_normal(h),
                w1=rng.standard_normal(h * m) * 0.05, b1=0.1 * rng.standard_normal(m),
                w2=rng.standard_normal(m * h) * 0.05, b2=0.1 * rng.standard_normal(h),
                ln2_gamma=1 + 0.1 * rng.standard_normal(h), ln2_beta=0.1 * rng.standard_normal(h))


@pytest.mark.parametrize("h,m,n", [(256, 512, 16), (200, 333, 7), (768, 3072, 33)])
def test_transformer_block_demo_forward(gae, ora, h, m, n):
    """ate::TransformerBlock::forward (transformer.rs:87-120) in fp32 through
    gae_transformer_block_forward_f32_host against the oracle's restatement:
    max-abs error <= 1e-5 of the output's largest value (the sums and
    LayerNorms follow the crate's order exactly; only tanh's last place in
    GELU may differ)."""
    cfg = gae.TransformerConfig(hidden_dim=h, num_heads=4, head_dim=h // 4, mlp_dim=m, eps=1e-5)
    rng = np.random.default_rng(h + m)
    w = {k_: v_.astype(np.float32) for k_, v_ in _crate_weights(rng, h, m).items()}
    block = gae.TransformerBlock(cfg, **w)
    x = rng.standard_normal(n * h).astype(np.float32)
    got = block.forward(x, n)
    ref = ora.transformer_block_forward(x, n, h, m, 1e-5, w["wv"], w["wo"], w["ln1_gamma"],
                                        w["ln1_beta"], w["w1"], w["b1"], w["w2"], w["b2"],
                                        w["ln2_gamma"], w["ln2_beta"])
    assert got.shape == ref.shape
    assert _rel(got, ref) <= 1e-5
    # new_random (constant weights) gives finite outputs of the right shape
    nb = gae.TransformerBlock.new_random(cfg)
    out = nb.forward(np.full(n * h, 0.1, np.float32), n)
    assert out.shape == (n * h,) and np.all(np.isfinite(out))


@pytest.mark.parametrize("h,m,t", [(256, 512, 3), (100, 250, 5), (768, 3072, 2)])
def test_crate_layer_primitives(gae, ora, h, m, t):
    """ate::layernorm / layernorm_batched / mlp_block / fused_mlp_layernorm
    (layernorm.rs, mlp.rs) through the fp32 host entry points against the
    oracle's restatement of the crate: LayerNorm bit-identical (same Welford
    order, IEEE division and square root), the MLPs within 1e-5 of the
    output's largest value (tanh's last place in GELU), any widths."""
    rng = np.random.default_rng(4 + h)
    x = rng.standard_normal(t * h).astype(np.float32)
    r = rng.standard_normal(t * h).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(h)).astype(np.float32)
    b = (0.1 * rng.standard_normal(h)).astype(np.float32)
    w1 = (rng.standard_normal(h * m) * 0.05).astype(np.float32)
    b1 = (0.1 * rng.standard_normal(m)).astype(np.float32)
    w2 = (rng.standard_normal(m * h) * 0.05).astype(np.float32)
    b2 = (0.1 * rng.standard_normal(h)).astype(np.float32)
    assert np.array_equal(gae.layernorm(x[:h], g, b, 1e-5), ora.layernorm(x[:h], g, b, 1e-5))
    assert np.array_equal(gae.layernorm_batched(x, g, b, t, h, 1e-5),
                          ora.layernorm_batched(x, g, b, t, h, 1e-5))
    for i in range(t):  # the crate's functions take one token
        sl = slice(i * h, (i + 1) * h)
        assert _rel(gae.mlp_block(x[sl], w1, b1, w2, b2, h, m),
                    ora.mlp_block(x[sl], w1, b1, w2, b2, h, m)) <= 1e-5
        assert _rel(gae.fused_mlp_layernorm(x[sl], r[sl], w1, b1, w2, b2, g, b, h, m, 1e-5),
                    ora.fused_mlp_layernorm(x[sl], r[sl], w1, b1, w2, b2, g, b, h, m, 1e-5)) <= 1e-5
    # several tokens at once give the same rows as one at a time
    many = gae.mlp_block(x, w1, b1, w2, b2, h, m)
    for i in range(t):
        sl = slice(i * h, (i + 1) * h)
        assert np.array_equal(many[sl], gae.mlp_block(x[sl], w1, b1, w2, b2, h, m))


def test_crate_linear_is_the_sequential_sum(gae, ora):
    """Without GELU the MLP's second product is a plain sum: the device
    linear kernel reproduces the crate's sequential f32 sum bit for bit
    (mlp.rs:26-31 order: bias first, then j = 0, 1, ...)."""
    rng = np.random.default_rng(11)
    M, N, K = 37, 130, 301
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.standard_normal((K, N)).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    y = torch.empty(M, N, device="cuda")
    xd, wd, bd = (torch.from_numpy(a).cuda() for a in (x, w, b))
    gae._check(gae.lib().gae_crate_linear_f32(xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), None,
                                             y.data_ptr(), M, N, K, 1, 0, None))
    ref = np.empty((M, N), np.float32)
    for i in range(N):  # sequential f32 sum, no contraction (numpy float32 scalars)
        s = b[i].copy() + np.zeros(M, np.float32)
        for j in range(K):
            s = (s + x[:, j] * w[j, i]).astype(np.float32)
        ref[:, i] = s
    assert np.array_equal(y.cpu().numpy(), ref)


def test_layernorm_kat_through_c_abi(gae):
    """tests/validation.rs:64-77 (test_layernorm_unit) through
    gae_layernorm_f32_host: LN([1, 2, 3, 4]) has mean 0 (1e-4) and variance
    1 (1e-2)."""
    out = gae.layernorm(np.array([1, 2, 3, 4], np.float32), np.ones(4, np.float32),
                        np.zeros(4, np.float32), 1e-5)
    mean = float(out.mean())
    assert abs(mean) <= 1e-4
    assert abs(float(((out - mean) ** 2).mean()) - 1.0) <= 1e-2
