"""Ulysses attention on the CUDA path (all-to-all over NCCL, one fused
attention launch per rank over the full sequence of its heads).  With one GPU
the P=1 path is the plain kernel; with two or more visible, NCCL ranks run
the exchange.  Tolerance: bf16 output within 2e-2 max-abs of the fp32 oracle."""
import math
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _inputs(B, H, N, D, seed=11):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, H, N, D, generator=g).bfloat16() for _ in range(3)]


def test_ulysses_single_gpu(gae, ora):
    from gae_b200 import ulysses
    q, k, v = _inputs(1, 4, 512, 128)
    o = ulysses.ulysses_attention(q.cuda(), k.cuda(), v.cuda(), causal=True)
    ref = ora.attention_batched(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                1 / math.sqrt(128), True)
    assert float(np.abs(o.float().cpu().numpy() - ref).max()) <= 2e-2


def test_ulysses_backward_single_gpu(gae, ora):
    """P=1 Ulysses backward (one gae_attn_bwd over the whole sequence) against
    the oracle's gradients; tolerance 2e-2 of each gradient's largest value."""
    from gae_b200 import ulysses
    q, k, v = _inputs(1, 4, 512, 128)
    do = _inputs(1, 4, 512, 128, seed=12)[0]
    qd, kd, vd, dod = (t.cuda() for t in (q, k, v, do))
    o, lse = ulysses.ulysses_attention(qd, kd, vd, causal=True, return_lse=True)
    grads = ulysses.ulysses_attention_backward(qd, kd, vd, o, dod, lse, causal=True)
    torch.cuda.synchronize()
    f = lambda t: t.float().cpu().numpy().reshape(4, 512, 128)
    refs = ora.attention_bwd(f(q), f(k), f(v), f(do), 1 / math.sqrt(128), True)
    for got, ref in zip(grads, refs):
        assert float(np.abs(f(got) - ref).max() / np.abs(ref).max()) <= 2e-2


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    import __graft_entry__ as ge
    ge.load_package()
    from gae_b200 import ulysses
    H = 2 * world
    q, k, v = _inputs(1, H, 256 * world, 128)
    S = 256
    sl = slice(rank * S, (rank + 1) * S)
    do = _inputs(1, H, 256 * world, 128, seed=12)[0]
    qs, ks, vs, dos = (t[:, :, sl].cuda() for t in (q, k, v, do))
    o, lse = ulysses.ulysses_attention(qs, ks, vs, causal=True, return_lse=True)
    grads = ulysses.ulysses_attention_backward(qs, ks, vs, o, dos, lse, causal=True)
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"o{rank}.npy"), o.float().cpu().numpy())
    for name, t in zip(("dq", "dk", "dv"), grads):
        np.save(os.path.join(out_dir, f"{name}{rank}.npy"), t.float().cpu().numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_ulysses_multi_gpu(ora, tmp_path):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True)
    q, k, v = _inputs(1, 2 * world, 256 * world, 128)
    ref = ora.attention_batched(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                1 / math.sqrt(128), True)
    got = np.concatenate([np.load(tmp_path / f"o{r}.npy") for r in range(world)], axis=2)
    assert float(np.abs(got - ref).max()) <= 2e-2
    do = _inputs(1, 2 * world, 256 * world, 128, seed=12)[0]
    f = lambda t: t.float().numpy().reshape(2 * world, 256 * world, 128)
    refs = ora.attention_bwd(f(q), f(k), f(v), f(do), 1 / math.sqrt(128), True)
    for name, r in zip(("dq", "dk", "dv"), refs):
        g = np.concatenate([np.load(tmp_path / f"{name}{i}.npy") for i in range(world)], axis=2)
        assert float(np.abs(g.reshape(r.shape) - r).max() / np.abs(r).max()) <= 2e-2, name
