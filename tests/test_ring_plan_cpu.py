"""Host logic of the C-ABI ring (gae_ring_attn_fwd), without GPUs or NCCL.

gae_debug_ring_plan returns the attention launches a rank issues at each ring
step.  Mapping each launch's buffer rows back to sequence positions (zig-zag:
rank r holds chunks r and 2P-1-r; contiguous: chunk r), every launch's mask
must equal the true causal relation of those positions, and over all steps
every visible (query, key) pair of every rank must be computed exactly once.
Also: the library loads on a CPU-only host and exports the ring entry points.
"""
import ctypes as C

import numpy as np
import pytest


def _plan(gae, rank, world, step, causal, zig, S):
    ops = (C.c_int64 * 14)()
    n = C.c_int()
    gae._check(gae.lib().gae_debug_ring_plan(rank, world, step, int(causal), int(zig), S, ops, C.byref(n)))
    return [tuple(ops[7 * i:7 * i + 7]) for i in range(n.value)]


def _positions(rank, world, zig, S):
    """Sequence position of each row of a rank's buffer (and of its K/V block)."""
    if zig:
        C_ = S // 2
        return np.concatenate([rank * C_ + np.arange(C_), (2 * world - 1 - rank) * C_ + np.arange(C_)])
    return rank * S + np.arange(S)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("causal,zig", [(True, True), (True, False), (False, False)])
def test_ring_plan_covers_each_visible_pair_once(gae, world, causal, zig):
    if zig and world == 1:
        pytest.skip("one rank runs one launch, no re-deal")
    S = 8
    N = S * world
    for r in range(world):
        qpos = _positions(r, world, zig, S)
        count = np.zeros((S, N), np.int64)  # per buffer row: how often each key was visited
        for t in range(world):
            src = (r - t) % world
            kpos = _positions(src, world, zig, S)
            for (q0, nq, k0, nk, caus, qp, kp) in _plan(gae, r, world, t, causal, zig, S):
                rows = np.arange(q0, q0 + nq)
                keys = np.arange(k0, k0 + nk)
                true_vis = kpos[keys][None, :] <= qpos[rows][:, None] if causal else \
                    np.ones((nq, nk), bool)
                if caus:
                    plan_vis = (kp + np.arange(nk))[None, :] <= (qp + np.arange(nq))[:, None]
                else:
                    plan_vis = np.ones((nq, nk), bool)
                assert np.array_equal(plan_vis, true_vis), (r, t)
                count[np.ix_(rows, kpos[keys])] += plan_vis
        want = (np.arange(N)[None, :] <= qpos[:, None]) if causal else np.ones((S, N), bool)
        assert np.array_equal(count, want.astype(np.int64)), r


def test_ring_plan_zigzag_balances_work(gae):
    """Zig-zag: after the diagonal step every rank computes the same number
    of (query, key) pairs per step."""
    world, S = 4, 16
    for t in range(1, world):
        work = {sum(nq * nk for (_, nq, _, nk, *_rest) in _plan(gae, r, world, t, True, True, S))
                for r in range(world)}
        assert len(work) == 1, (t, work)


def test_ring_entry_points_exported(gae):
    L = gae.lib()
    for name in ("gae_ring_unique_id", "gae_ring_ctx_create", "gae_ring_ctx_create_from_comm",
                 "gae_ring_attn_fwd", "gae_ring_ctx_destroy"):
        assert hasattr(L, name)
    # argument checks run on the host, without a context or a GPU
    with pytest.raises(gae.GAEError):
        gae._check(L.gae_ring_attn_fwd(None, None, 0, None))
