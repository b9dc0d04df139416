"""Pins the CPU oracle (oracle/gae_oracle.c) against the reference's own
known-answer tests (tests/validation.rs in the reference project) and against
the committed golden fixture, before the oracle is trusted as the checker of
the CUDA kernels.  CPU only."""
import math

import numpy as np
import pytest


def close(a, b, eps):
    # approx::assert_relative_eq!(a, b, epsilon = eps): |a-b| <= eps or relative
    return abs(a - b) <= eps or abs(a - b) <= eps * max(abs(a), abs(b))


# tests/validation.rs:6-15
def test_welford_mean_variance(ora):
    w = ora.WelfordState()
    for x in [2.0, 4.0, 4.0, 4.0, 5.0, 5.0, 7.0, 9.0]:
        w.update(x)
    assert close(w.mean, 5.0, 1e-5)
    assert close(w.variance(), 4.0, 1e-5)


# tests/validation.rs:17-36
def test_welford_merge(ora):
    a, b, full = ora.WelfordState(), ora.WelfordState(), ora.WelfordState()
    for x in [1.0, 2.0, 3.0, 4.0]:
        a.update(x); full.update(x)
    for x in [5.0, 6.0, 7.0, 8.0]:
        b.update(x); full.update(x)
    m = ora.WelfordState.merge(a, b)
    assert close(m.mean, full.mean, 1e-5)
    assert close(m.variance(), full.variance(), 1e-5)


# tests/validation.rs:38-55
def test_online_softmax_equivalence(ora):
    scores = [1.0, 2.0, 3.0, 4.0, 5.0]
    s = ora.OnlineSoftmax()
    for x in scores:
        s.update(x)
    mx = max(scores)
    z = sum(math.exp(x - mx) for x in scores)
    for x in scores:
        assert close(s.probability(x), math.exp(x - mx) / z, 1e-5)


# tests/validation.rs:57-62
def test_gelu_values(ora):
    assert close(ora.gelu(0.0), 0.0, 1e-5)
    assert close(ora.gelu(1.0), 0.8413, 1e-3)
    assert close(ora.gelu(-1.0), -0.1587, 1e-3)


# tests/validation.rs:64-77
def test_layernorm_unit(ora):
    out = ora.layernorm(np.array([1, 2, 3, 4], np.float32), np.ones(4), np.zeros(4), 1e-5)
    mean = float(out.mean())
    var = float(((out - mean) ** 2).mean())
    assert close(mean, 0.0, 1e-4)
    assert close(var, 1.0, 1e-2)


# tests/validation.rs:79-94
def test_waller_operator_causal(ora):
    n, d = 4, 2
    q = np.ones(n * d, np.float32); k = np.ones(n * d, np.float32)
    v = np.arange(n * d, dtype=np.float32)
    out = ora.waller_operator(q, k, v, n, d, 1.0 / math.sqrt(d))
    assert out.size == n * d
    assert close(out[0], v[0], 1e-4) and close(out[1], v[1], 1e-4)


# tests/validation.rs:96-114 (the demo forward: shapes and finiteness)
def test_transformer_block_shapes(ora):
    h, m, n = 64, 256, 8
    const = lambda size, val: np.full(size, val, np.float32)
    out = ora.transformer_block_forward(
        const(n * h, 0.1), n, h, m, 1e-5, const(h * h, 0.02), const(h * h, 0.02),
        const(h, 1.0), const(h, 0.0), const(h * m, 0.02), const(m, 0.0), const(m * h, 0.02),
        const(h, 0.0), const(h, 1.0), const(h, 0.0))
    assert out.size == n * h
    assert np.all(np.isfinite(out))


# tests/validation.rs:129-145
def test_standard_attention_causal(ora):
    n, d = 4, 2
    q = np.ones(n * d, np.float32); k = np.ones(n * d, np.float32)
    v = np.arange(n * d, dtype=np.float32)
    out = ora.standard_attention(q, k, v, n, d, 1.0 / math.sqrt(d))
    assert close(out[0], v[0], 1e-4) and close(out[1], v[1], 1e-4)


# tests/validation.rs:147-163
def test_standard_vs_waller_equivalence(ora):
    n, d = 16, 8
    i = np.arange(n * d, dtype=np.float32)
    q = np.sin(i * np.float32(0.1)); k = np.cos(i * np.float32(0.2)); v = np.sin(i * np.float32(0.05))
    st = ora.standard_attention(q, k, v, n, d, 1.0 / math.sqrt(d))
    wa = ora.waller_operator(q, k, v, n, d, 1.0 / math.sqrt(d))
    for a, b in zip(st, wa):
        assert close(float(a), float(b), 1e-4)


def test_parallel_matches_sequential_bitwise(ora):
    rng = np.random.default_rng(5)
    n, d = 200, 64
    q, k, v = (rng.standard_normal(n * d).astype(np.float32) for _ in range(3))
    for causal in (True, False):
        a = ora.waller_operator(q, k, v, n, d, 0.125, causal=causal)
        b = ora.waller_operator(q, k, v, n, d, 0.125, causal=causal, parallel=True)
        assert np.array_equal(a, b)


def _ref64(q, k, v, scale, causal):
    s = (q.astype(np.float64) @ k.astype(np.float64).T) * scale
    if causal:
        s = np.where(np.tril(np.ones_like(s, dtype=bool)), s, -np.inf)
    s -= s.max(axis=1, keepdims=True)
    p = np.exp(s)
    return (p / p.sum(axis=1, keepdims=True)) @ v.astype(np.float64)


@pytest.mark.parametrize("causal", [True, False])
def test_config1_against_float64(ora, causal):
    """N=1024, d=64, iid N(0,1) from a fixed seed."""
    from tests.golden.make_golden import config1_inputs
    q, k, v = config1_inputs()
    out = ora.waller_operator(q, k, v, 1024, 64, 1.0 / 8.0, causal=causal).reshape(1024, 64)
    ref = _ref64(q, k, v, 1.0 / 8.0, causal)
    # fp32 tolerance: 1e-5 relative to the tensor's scale (max-abs error over
    # max |ref|) and 1e-5 relative L2.
    assert np.abs(out - ref).max() / np.abs(ref).max() < 1e-5
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) < 1e-5


@pytest.mark.parametrize("causal", [True, False])
def test_config1_golden_fixture(ora, causal):
    from tests.golden.make_golden import config1_inputs, load_golden
    q, k, v = config1_inputs()
    rows, expect = load_golden("config1_causal" if causal else "config1_noncausal")
    out = ora.waller_operator(q, k, v, 1024, 64, 1.0 / 8.0, causal=causal).reshape(1024, 64)
    assert np.abs(out[rows] - expect).max() / np.abs(expect).max() < 1e-5


def test_batched_offsets_match_single(ora):
    rng = np.random.default_rng(1)
    B, H, N, D = 1, 2, 96, 32
    q, k, v = (rng.standard_normal((B, H, N, D)).astype(np.float32) for _ in range(3))
    full = ora.attention_batched(q, k, v, 0.2, True)
    # Query block [48, 96) against key block [0, 48) and [48, 96), merged by LSE.
    o1, l1 = ora.attention_batched(q[:, :, 48:], k[:, :, :48], v[:, :, :48], 0.2, True,
                                   q_offset=48, kv_offset=0, want_lse=True)
    o2, l2 = ora.attention_batched(q[:, :, 48:], k[:, :, 48:], v[:, :, 48:], 0.2, True,
                                   q_offset=48, kv_offset=48, want_lse=True)
    om, _ = ora.lse_merge(o1, l1, o2, l2)
    assert np.abs(om - full[:, :, 48:]).max() < 1e-5


def test_int8_quantize_and_logits(ora):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((4, 64)).astype(np.float32)
    q, s = ora.quantize_rows_int8(x)
    assert np.abs(q).max() == 127
    assert np.allclose(q * s[:, None], x, atol=s.max())
    L = ora.int8_logits(q[None], q[None])
    assert np.array_equal(L[0], q.astype(np.int32) @ q.astype(np.int32).T)


def test_attention_bwd_oracle_matches_autograd(ora):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(3)
    for causal, (n, m) in ((True, (37, 37)), (False, (29, 41))):
        q, g = (rng.standard_normal((2, n, 16)).astype(np.float32) for _ in range(2))
        k, v = (rng.standard_normal((2, m, 16)).astype(np.float32) for _ in range(2))
        dq, dk, dv = ora.attention_bwd(q, k, v, g, 0.3, causal)
        Q, K, V = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (q, k, v))
        s = Q @ K.transpose(1, 2) * 0.3
        if causal:
            s = s.masked_fill(torch.triu(torch.ones(n, m, dtype=torch.bool), 1), float("-inf"))
        (torch.softmax(s, -1) @ V).backward(torch.tensor(g, dtype=torch.float64))
        for got, t in ((dq, Q), (dk, K), (dv, V)):
            assert np.abs(got - t.grad.numpy()).max() < 1e-5
