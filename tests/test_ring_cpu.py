"""Ring-attention host logic on CPU ranks (gloo, world sizes 2 and 3).

The block compute is injected: the oracle's batched Waller recurrence plays
the kernel and its LSE merge plays gae_lse_merge, so the test checks the
driver's ring schedule, causal block skipping, zig-zag re-dealing and merge
bookkeeping against one full-sequence oracle call.  The CUDA path of the same
driver is covered by tests/test_ring_gpu.py.
"""
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_attend(q, k, v, causal, q_offset, kv_offset, scale):
    from oracle import oracle
    o, lse = oracle.attention_batched(q.float().contiguous().numpy(), k.float().contiguous().numpy(),
                                      v.float().contiguous().numpy(), scale, causal,
                                      q_offset=q_offset, kv_offset=kv_offset, want_lse=True)
    return torch.from_numpy(o), torch.from_numpy(lse)


def _oracle_merge(o_acc, lse_acc, o_part, lse_part):
    from oracle import oracle
    o, l = oracle.lse_merge(o_acc.numpy(), lse_acc.numpy(), o_part.float().numpy(),
                            lse_part.numpy())
    o_acc.copy_(torch.from_numpy(o))
    lse_acc.copy_(torch.from_numpy(l))


def _worker(rank, world, port, causal, balance, result_dir):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import __graft_entry__ as ge
    gae = ge.load_package()
    from gae_b200 import ring
    B, H, S, D = 1, 2, 8, 16
    g = torch.Generator().manual_seed(42)
    full = [torch.randn(B, H, S * world, D, generator=g) for _ in range(3)]
    q, k, v = (t[:, :, rank * S:(rank + 1) * S].contiguous() for t in full)
    o, lse = ring.ring_attention(q, k, v, causal=causal, balance=balance, return_lse=True,
                                 attend=_oracle_attend, merge=_oracle_merge)
    np.save(os.path.join(result_dir, f"o{rank}.npy"), o.numpy())
    np.save(os.path.join(result_dir, f"l{rank}.npy"), lse.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("causal,balance", [(True, "zigzag"), (True, "contiguous"),
                                            (False, "contiguous")])
def test_ring_matches_full_attention(tmp_path, ora, world, causal, balance):
    port = _free_port()
    mp.spawn(_worker, args=(world, port, causal, balance, str(tmp_path)), nprocs=world, join=True)
    B, H, S, D = 1, 2, 8, 16
    g = torch.Generator().manual_seed(42)
    full = [torch.randn(B, H, S * world, D, generator=g) for _ in range(3)]
    ref, rlse = ora.attention_batched(*(t.numpy() for t in full), 1 / math.sqrt(D), causal,
                                      want_lse=True)
    got = np.concatenate([np.load(tmp_path / f"o{r}.npy") for r in range(world)], axis=2)
    gl = np.concatenate([np.load(tmp_path / f"l{r}.npy") for r in range(world)], axis=2)
    assert np.abs(got - ref).max() < 1e-5
    assert np.abs(gl - rlse).max() < 1e-5


def test_zigzag_owner_is_a_balanced_partition():
    import __graft_entry__ as ge
    ge.load_package()
    from gae_b200 import ring
    for P in (1, 2, 4, 8):
        owners = [ring.zigzag_owner(c, P) for c in range(2 * P)]
        assert sorted(owners) == sorted(list(range(P)) * 2)
        for r in range(P):
            mine = [c for c in range(2 * P) if owners[c] == r]
            assert mine == [r, 2 * P - 1 - r]


def _block_bwd(q, k, v, out, dout, lse, causal, scale):
    """One block pair's share of the gradients given the final output and LSE
    of its query rows (what gae_attn_bwd computes), in float64."""
    q, k, v, out, dout, lse = (t.double() for t in (q, k, v, out, dout, lse))
    s = q @ k.transpose(-1, -2) * scale
    if causal:
        n, m = s.shape[-2:]
        s = s.masked_fill(torch.triu(torch.ones(n, m, dtype=torch.bool), 1), float("-inf"))
    p = torch.exp(s - lse.unsqueeze(-1))
    dv = p.transpose(-1, -2) @ dout
    dp = dout @ v.transpose(-1, -2)
    ds = p * (dp - (dout * out).sum(-1, keepdim=True))
    return ds @ k * scale, ds.transpose(-1, -2) @ q * scale, dv


def _bwd_worker(rank, world, port, causal, balance, result_dir):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import __graft_entry__ as ge
    ge.load_package()
    from gae_b200 import ring
    B, H, S, D = 1, 2, 8, 16
    g = torch.Generator().manual_seed(43)
    full = [torch.randn(B, H, S * world, D, generator=g) for _ in range(4)]
    q, k, v, do = (t[:, :, rank * S:(rank + 1) * S].contiguous() for t in full)
    o, lse = ring.ring_attention(q, k, v, causal=causal, balance=balance, return_lse=True,
                                 attend=_oracle_attend, merge=_oracle_merge)
    dq, dk, dv = ring.ring_attention_backward(q, k, v, o, do, lse, causal=causal, balance=balance,
                                              attend_bwd=_block_bwd)
    for name, t in (("dq", dq), ("dk", dk), ("dv", dv)):
        np.save(os.path.join(result_dir, f"{name}{rank}.npy"), t.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("causal,balance", [(True, "zigzag"), (True, "contiguous"),
                                            (False, "contiguous")])
def test_ring_backward_matches_full_gradients(tmp_path, ora, world, causal, balance):
    port = _free_port()
    mp.spawn(_bwd_worker, args=(world, port, causal, balance, str(tmp_path)), nprocs=world,
             join=True)
    B, H, S, D = 1, 2, 8, 16
    g = torch.Generator().manual_seed(43)
    full = [torch.randn(B, H, S * world, D, generator=g) for _ in range(4)]
    f = lambda t: t.numpy().reshape(B * H, S * world, D)
    refs = ora.attention_bwd(f(full[0]), f(full[1]), f(full[2]), f(full[3]), 1 / math.sqrt(D), causal)
    for name, ref in zip(("dq", "dk", "dv"), refs):
        got = np.concatenate([np.load(tmp_path / f"{name}{r}.npy") for r in range(world)], axis=2)
        assert np.abs(got.reshape(ref.shape) - ref).max() < 1e-4, name
