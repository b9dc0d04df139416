"""Parity of the CUDA attention kernels against the CPU oracle, through the C ABI.

Tolerances (written here, as the benchmark plan states them):
  fp32 path: max-abs error <= 1e-5 x max|ref| and relative L2 <= 1e-5 against
             the fp32 oracle on identical inputs;
  bf16/f16:  max-abs error <= 2e-2 against the fp32 oracle fed the same
             bf16-rounded inputs; log-sum-exp within 1e-3 absolute.
"""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


def rel_scale(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


# ---------------------------------------------------------------- fp32 path
@pytest.mark.parametrize("causal", [True, False])
def test_config1_f32_host_dropin(gae, ora, causal):
    from tests.golden.make_golden import config1_inputs, load_golden
    q, k, v = config1_inputs()
    out = gae.waller_operator(q, k, v, 1024, 64, 0.125, causal=causal).reshape(1024, 64)
    ref = ora.waller_operator(q, k, v, 1024, 64, 0.125, causal=causal).reshape(1024, 64)
    assert rel_scale(out, ref) <= 1e-5
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) <= 1e-5
    rows, gold = load_golden("config1_causal" if causal else "config1_noncausal")
    assert rel_scale(out[rows], gold) <= 1e-5
    # the elementwise-relative form (floor 1e-3 of the largest output)
    assert elementwise_rel(out, ref) <= 1e-3


def elementwise_rel(a, b):
    """max |a - b| / max(|b|, 1e-3 max|b|): the elementwise-relative fp32
    metric (tighter than rel_scale on small outputs)."""
    b_abs = np.abs(b)
    return float((np.abs(a - b) / np.maximum(b_abs, 1e-3 * b_abs.max())).max())


@pytest.mark.parametrize("n,d,causal", [(1024, 64, True), (1024, 64, False), (333, 40, True),
                                        (96, 256, False)])
def test_standard_attention_against_oracle(gae, ora, n, d, causal):
    """ate::standard_attention (standard_attention.rs:13-65) through
    gae_standard_attention_f32_host against the oracle's restatement of the
    materialised N x N form (not against the library's own Waller path):
    1e-5 of the output's scale and 1e-5 relative L2; the elementwise-relative
    error is bounded too."""
    rng = np.random.default_rng(n + d)
    q, k, v = (rng.standard_normal(n * d).astype(np.float32) for _ in range(3))
    scale = 1.0 / math.sqrt(d)
    got = gae.standard_attention(q, k, v, n, d, scale, causal=causal)
    ref = ora.standard_attention(q, k, v, n, d, scale, causal=causal)
    assert rel_scale(got, ref) <= 1e-5
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-5
    assert elementwise_rel(got, ref) <= 1e-3


def test_reference_kats_on_gpu(gae):
    # tests/validation.rs:79-94 through the GPU drop-in
    n, d = 4, 2
    v = np.arange(n * d, dtype=np.float32)
    out = gae.waller_operator(np.ones(n * d), np.ones(n * d), v, n, d, 1 / math.sqrt(d))
    assert abs(out[0] - v[0]) <= 1e-4 and abs(out[1] - v[1]) <= 1e-4
    # tests/validation.rs:147-163
    n, d = 16, 8
    i = np.arange(n * d, dtype=np.float32)
    q = np.sin(i * np.float32(0.1)); k = np.cos(i * np.float32(0.2)); vv = np.sin(i * np.float32(0.05))
    st = gae.standard_attention(q, k, vv, n, d, 1 / math.sqrt(d))
    wa = gae.waller_operator_parallel(q, k, vv, n, d, 1 / math.sqrt(d))
    assert np.abs(st - wa).max() <= 1e-4


def test_f32_device_batched_offsets(gae, ora):
    g = torch.Generator().manual_seed(3)
    B, H, Nq, Nkv, D = 2, 3, 200, 330, 96
    q = torch.randn(B, H, Nq, D, generator=g)
    k = torch.randn(B, H, Nkv, D, generator=g)
    v = torch.randn(B, H, Nkv, D, generator=g)
    o, lse = gae.attention(q.cuda(), k.cuda(), v.cuda(), causal=True, q_offset=130, kv_offset=0,
                           return_lse=True)
    ref, rlse = ora.attention_batched(q.numpy(), k.numpy(), v.numpy(), 1 / math.sqrt(D), True,
                                      q_offset=130, want_lse=True)
    assert rel_scale(o.cpu().numpy(), ref) <= 1e-5
    assert np.abs(lse.cpu().numpy() - rlse).max() <= 1e-5


def test_f32_host_rejects_short_input(gae):
    with pytest.raises(gae.GAEError):
        gae.waller_operator(np.ones(7), np.ones(8), np.ones(8), 4, 2, 1.0)


# ---------------------------------------------------------- tensor-core path
def _rand(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype)


def _check_tc(gae, ora, B, H, Nq, Nkv, D, causal, dtype=torch.bfloat16, q_offset=0,
              kv_offset=0, layout="bhsd", seed=0):
    q = _rand((B, H, Nq, D), dtype, seed)
    k = _rand((B, H, Nkv, D), dtype, seed + 1)
    v = _rand((B, H, Nkv, D), dtype, seed + 2)
    if layout == "bshd":  # strided views of [B, N, H, D] storage
        qd = q.transpose(1, 2).contiguous().cuda().transpose(1, 2)
        kd = k.transpose(1, 2).contiguous().cuda().transpose(1, 2)
        vd = v.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    else:
        qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    o, lse = gae.attention(qd, kd, vd, causal=causal, q_offset=q_offset, kv_offset=kv_offset,
                           return_lse=True)
    torch.cuda.synchronize()
    gae.device_status()
    ref, rlse = ora.attention_batched(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                      1 / math.sqrt(D), causal, q_offset=q_offset,
                                      kv_offset=kv_offset, want_lse=True)
    got = o.float().cpu().numpy()
    err = float(np.abs(got - ref).max())
    assert err <= BF16_TOL, f"max-abs {err}"
    gl = lse.cpu().numpy()
    fin = np.isfinite(rlse)
    assert np.array_equal(np.isfinite(gl), fin)
    if fin.any():
        assert np.abs(gl[fin] - rlse[fin]).max() <= 1e-3
    return o


@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("causal", [False, True])
def test_tc_square(gae, ora, D, causal):
    _check_tc(gae, ora, 1, 2, 512, 512, D, causal)


@pytest.mark.parametrize("N", [1, 100, 128, 129, 255, 256, 257, 777])
def test_tc_ragged_lengths(gae, ora, N):
    _check_tc(gae, ora, 1, 2, N, N, 128, True, seed=N)
    _check_tc(gae, ora, 1, 1, N, N, 64, False, seed=N + 7)


def test_tc_cross_lengths(gae, ora):
    _check_tc(gae, ora, 2, 2, 300, 1000, 128, False)
    _check_tc(gae, ora, 1, 3, 1000, 300, 64, False)


def test_tc_strided_bshd_layout(gae, ora):
    _check_tc(gae, ora, 2, 4, 384, 384, 128, True, layout="bshd")


def test_tc_fp16(gae, ora):
    _check_tc(gae, ora, 1, 2, 384, 384, 128, True, dtype=torch.float16)


@pytest.mark.parametrize("causal", [True, False])
def test_tc_fp16_head_dim_64(gae, ora, causal):
    """f16 at head_dim 64 (the tensor-core row sums read an f16 panel of
    ones), ragged length."""
    _check_tc(gae, ora, 2, 3, 333, 333, 64, causal, dtype=torch.float16)


@pytest.mark.parametrize("q_offset,kv_offset", [(512, 0), (512, 256), (0, 512), (100, 37)])
def test_tc_ring_block_offsets(gae, ora, q_offset, kv_offset):
    # A query block attending to one key block of a longer causal sequence.
    _check_tc(gae, ora, 1, 2, 256, 256, 128, True, q_offset=q_offset, kv_offset=kv_offset)


def test_tc_large_scores_rescale(gae, ora):
    # Scores spread over a wide range exercise the lazy max rescaling.
    B, H, N, D = 1, 1, 1024, 128
    q = _rand((B, H, N, D), torch.float32, 9) * 4
    k = _rand((B, H, N, D), torch.float32, 10) * 4
    v = _rand((B, H, N, D), torch.float32, 11)
    qb, kb, vb = q.bfloat16(), k.bfloat16(), v.bfloat16()
    o = gae.attention(qb.cuda(), kb.cuda(), vb.cuda(), causal=True)
    ref = ora.attention_batched(qb.float().numpy(), kb.float().numpy(), vb.float().numpy(),
                                1 / math.sqrt(D), True)
    assert float(np.abs(o.float().cpu().numpy() - ref).max()) <= BF16_TOL


def test_tc_deterministic(gae):
    q, k, v = (_rand((2, 4, 1024, 128), torch.bfloat16, s).cuda() for s in (1, 2, 3))
    a = gae.attention(q, k, v, causal=True)
    b = gae.attention(q, k, v, causal=True)
    assert torch.equal(a, b)


def test_tc_matches_torch_sdpa(gae):
    # Cross-check against PyTorch's own attention at a mid size.
    q, k, v = (_rand((2, 8, 2048, 128), torch.bfloat16, s).cuda() for s in (4, 5, 6))
    for causal in (False, True):
        o = gae.attention(q, k, v, causal=causal)
        r = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(),
                                                             is_causal=causal)
        assert float((o.float() - r).abs().max()) <= BF16_TOL


def test_tc_rejects_bad_head_dim(gae):
    q = torch.zeros(1, 1, 128, 96, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(gae.GAEError):
        gae.attention(q, q, q)


def test_tc_empty_query(gae):
    q = torch.zeros(1, 1, 0, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(1, 1, 128, 128, dtype=torch.bfloat16, device="cuda")
    o = gae.attention(q, k, k)
    assert o.shape == (1, 1, 0, 128)


def test_lse_merge_matches_oracle(gae, ora):
    g = torch.Generator().manual_seed(8)
    rows, D = 1000, 128
    o1 = torch.randn(rows, D, generator=g); o2 = torch.randn(rows, D, generator=g)
    l1 = torch.randn(rows, generator=g) * 3; l2 = torch.randn(rows, generator=g) * 3
    l2[:10] = -float("inf")
    ro, rl = ora.lse_merge(o1.numpy(), l1.numpy(), o2.numpy(), l2.numpy())
    a, la = o1.cuda(), l1.cuda()
    gae.lse_merge_(a, la, o2.cuda(), l2.cuda())
    assert rel_scale(a.cpu().numpy(), ro) <= 1e-5
    assert np.abs(la.cpu().numpy() - rl).max() <= 1e-5
    b1, b2 = o1.bfloat16(), o2.bfloat16()
    rbo, _ = ora.lse_merge(b1.float().numpy(), l1.numpy(), b2.float().numpy(), l2.numpy())
    ab = b1.cuda()
    gae.lse_merge_(ab, l1.clone().cuda(), b2.cuda(), l2.cuda())
    assert float(np.abs(ab.float().cpu().numpy() - rbo).max()) <= BF16_TOL


def test_quantize_rows_int8_bit_exact(gae, ora):
    x = _rand((64, 128), torch.float32, 12)
    x[3] = 0
    q, s = gae.quantize_rows_int8(x.cuda())
    rq, rs = ora.quantize_rows_int8(x.numpy())
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(s.cpu().numpy(), rs)
    xb = x.bfloat16()
    q, s = gae.quantize_rows_int8(xb.cuda())
    rq, rs = ora.quantize_rows_int8(xb.float().numpy())
    assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tc_scores_growing_along_keys(gae, ora, D, causal, dtype):
    """Keys whose scores grow along the sequence, so that a row's running max
    keeps rising by more than the lazy rescale's headroom from tile to tile:
    exercises the rebasing and the recomputation after a speculative tile."""
    B, H, N = 1, 2, 1024
    g = torch.Generator().manual_seed(21)
    q = torch.randn(B, H, N, D, generator=g).abs()
    k = torch.randn(B, H, N, D, generator=g).abs() * torch.linspace(0.1, 3.0, N).view(1, 1, N, 1)
    v = torch.randn(B, H, N, D, generator=g)
    q, k, v = (t.to(dtype) for t in (q, k, v))
    o, lse = gae.attention(q.cuda(), k.cuda(), v.cuda(), causal=causal, return_lse=True)
    torch.cuda.synchronize()
    gae.device_status()
    ref, rlse = ora.attention_batched(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                      1 / math.sqrt(D), causal, want_lse=True)
    assert float(np.abs(o.float().cpu().numpy() - ref).max()) <= BF16_TOL
    assert float(np.abs(lse.cpu().numpy() - rlse).max()) <= 1e-3 * max(1.0, float(np.abs(rlse).max()))


def test_ate_gpu_backend_api(gae, ora):
    """ate::gpu::AteGpu::{new, waller_operator} (the crate's wgpu backend API)
    on the CUDA fp32 path: causal, same tolerance as the fp32 path."""
    rng = np.random.default_rng(17)
    n, d = 300, 64
    q, k, v = (rng.standard_normal(n * d).astype(np.float32) for _ in range(3))
    out = gae.AteGpu.new().waller_operator(q, k, v, n, d, 1 / math.sqrt(d)).reshape(n, d)
    ref = ora.waller_operator(q, k, v, n, d, 1 / math.sqrt(d), causal=True).reshape(n, d)
    assert rel_scale(out, ref) <= 1e-5


def test_reference_waller_kernels_pin_oracle_and_product(gae, ora):
    """The reference's own fp32 Waller kernels (cuda_src/waller_operator.cu:
    12-100, built from its source into oracle/_ref) against the oracle's
    restatement and this library's fp32 and bf16 paths on the same inputs
    (fp32: max-abs <= 1e-5 of the largest output; bf16: 2e-2 max-abs)."""
    L = ora.ref_waller()
    if L is None:
        pytest.skip("reference Waller kernels not built (no reference tree where build() ran)")
    rng = np.random.default_rng(23)
    st = torch.cuda.current_stream().cuda_stream
    # single head [N, d], the reference's own layout
    n, d = 1000, 64
    q, k, v = (rng.standard_normal(n * d).astype(np.float32) for _ in range(3))
    qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, k, v))
    od = torch.empty_like(qd)
    assert L.ref_waller_operator_fwd(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), od.data_ptr(), n, d,
                                     0.125, st) == 0
    torch.cuda.synchronize()
    ref_gpu = od.cpu().numpy().reshape(n, d)
    assert rel_scale(ora.waller_operator(q, k, v, n, d, 0.125, causal=True).reshape(n, d), ref_gpu) <= 1e-5
    assert rel_scale(gae.waller_operator(q, k, v, n, d, 0.125).reshape(n, d), ref_gpu) <= 1e-5
    # multi-head [H, N, d]
    h, n, d = 4, 777, 128
    q, k, v = (rng.standard_normal((1, h, n, d)).astype(np.float32) for _ in range(3))
    qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, k, v))
    od = torch.empty_like(qd)
    scale = 1 / math.sqrt(d)
    assert L.ref_waller_operator_multihead_fwd(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), od.data_ptr(),
                                               n, d, h, scale, st) == 0
    torch.cuda.synchronize()
    ref_gpu = od.cpu().numpy()
    o32 = gae.attention(qd, kd, vd, causal=True)
    assert rel_scale(o32.cpu().numpy(), ref_gpu) <= 1e-5
    o16 = gae.attention(qd.bfloat16(), kd.bfloat16(), vd.bfloat16(), causal=True)
    ref16 = ora.attention_batched(*(t.bfloat16().float().cpu().numpy() for t in (qd, kd, vd)), scale, True)
    assert float(np.abs(o16.float().cpu().numpy() - ref16).max()) <= BF16_TOL
    assert float(np.abs(ref16 - ref_gpu).max()) <= 5e-2  # bf16 input rounding only
