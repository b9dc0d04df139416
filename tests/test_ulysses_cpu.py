"""Ulysses (head/sequence all-to-all) host logic on CPU gloo ranks, with the
oracle's batched Waller recurrence injected as the attention kernel, against
one full-sequence oracle call."""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _attend(q, k, v, causal, scale):
    from oracle import oracle
    return torch.from_numpy(oracle.attention_batched(q.contiguous().numpy(), k.contiguous().numpy(),
                                                     v.contiguous().numpy(), scale, causal))


def _worker(rank, world, port, causal, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import __graft_entry__ as ge
    ge.load_package()
    from gae_b200 import ulysses
    B, H, S, D = 2, 4, 8, 16
    g = torch.Generator().manual_seed(9)
    full = [torch.randn(B, H, S * world, D, generator=g) for _ in range(3)]
    q, k, v = (t[:, :, rank * S:(rank + 1) * S].contiguous() for t in full)
    o = ulysses.ulysses_attention(q, k, v, causal=causal, attend=_attend)
    np.save(os.path.join(out_dir, f"o{rank}.npy"), o.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("causal", [True, False])
def test_ulysses_matches_full_attention(tmp_path, ora, world, causal):
    mp.spawn(_worker, args=(world, _port(), causal, str(tmp_path)), nprocs=world, join=True)
    B, H, S, D = 2, 4, 8, 16
    g = torch.Generator().manual_seed(9)
    full = [torch.randn(B, H, S * world, D, generator=g) for _ in range(3)]
    ref = ora.attention_batched(*(t.numpy() for t in full), 1 / math.sqrt(D), causal)
    got = np.concatenate([np.load(tmp_path / f"o{r}.npy") for r in range(world)], axis=2)
    assert np.abs(got - ref).max() < 1e-5


def test_ulysses_rejects_indivisible_heads():
    import __graft_entry__ as ge
    ge.load_package()
    from gae_b200 import ulysses
    if not dist.is_initialized():
        q = torch.zeros(1, 3, 8, 16)
        # one rank: any head count works
        out = ulysses.ulysses_attention(q, q, q, attend=lambda q, k, v, c, s: q)
        assert out.shape == q.shape


def _attend_lse(q, k, v, causal, scale, return_lse=False):
    from oracle import oracle
    o, lse = oracle.attention_batched(q.contiguous().numpy(), k.contiguous().numpy(),
                                      v.contiguous().numpy(), scale, causal, want_lse=True)
    return (torch.from_numpy(o), torch.from_numpy(lse)) if return_lse else torch.from_numpy(o)


def _attend_bwd(q, k, v, out, dout, lse, causal, scale):
    """Gradients from the given output and LSE (what gae_attn_bwd computes), float64."""
    q, k, v, out, dout, lse = (t.double() for t in (q, k, v, out, dout, lse))
    s = q @ k.transpose(-1, -2) * scale
    if causal:
        n = s.shape[-1]
        s = s.masked_fill(torch.triu(torch.ones(n, n, dtype=torch.bool), 1), float("-inf"))
    p = torch.exp(s - lse.unsqueeze(-1))
    ds = p * (dout @ v.transpose(-1, -2) - (dout * out).sum(-1, keepdim=True))
    return ds @ k * scale, ds.transpose(-1, -2) @ q * scale, p.transpose(-1, -2) @ dout


def _bwd_worker(rank, world, port, causal, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import __graft_entry__ as ge
    ge.load_package()
    from gae_b200 import ulysses
    B, H, S, D = 2, 4, 8, 16
    g = torch.Generator().manual_seed(10)
    full = [torch.randn(B, H, S * world, D, generator=g) for _ in range(4)]
    q, k, v, do = (t[:, :, rank * S:(rank + 1) * S].contiguous() for t in full)
    o, lse = ulysses.ulysses_attention(q, k, v, causal=causal, attend=_attend_lse, return_lse=True)
    grads = ulysses.ulysses_attention_backward(q, k, v, o, do, lse, causal=causal,
                                               attend_bwd=_attend_bwd)
    np.save(os.path.join(out_dir, f"l{rank}.npy"), lse.numpy())
    for name, t in zip(("dq", "dk", "dv"), grads):
        np.save(os.path.join(out_dir, f"{name}{rank}.npy"), t.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("causal", [True, False])
def test_ulysses_backward_matches_full_gradients(tmp_path, ora, world, causal):
    mp.spawn(_bwd_worker, args=(world, _port(), causal, str(tmp_path)), nprocs=world, join=True)
    B, H, S, D = 2, 4, 8, 16
    g = torch.Generator().manual_seed(10)
    full = [torch.randn(B, H, S * world, D, generator=g) for _ in range(4)]
    _, rlse = ora.attention_batched(*(t.numpy() for t in full[:3]), 1 / math.sqrt(D), causal,
                                    want_lse=True)
    gl = np.concatenate([np.load(tmp_path / f"l{r}.npy") for r in range(world)], axis=2)
    assert np.abs(gl - rlse).max() < 1e-5
    f = lambda t: t.numpy().reshape(B * H, S * world, D)
    refs = ora.attention_bwd(*(f(t) for t in full), 1 / math.sqrt(D), causal)
    for name, ref in zip(("dq", "dk", "dv"), refs):
        got = np.concatenate([np.load(tmp_path / f"{name}{r}.npy") for r in range(world)], axis=2)
        assert np.abs(got.reshape(ref.shape) - ref).max() < 1e-4, name
