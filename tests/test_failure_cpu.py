"""Failure detection without a GPU fault (host side, CPU gloo ranks).

A rank that leaves before the ring exchange, or arrives only after the
process group's timeout, must make the surviving rank raise
GAEError(GAE_ERR_COMM) within the timeout instead of hanging.  The block
compute is the oracle, injected as in tests/test_ring_cpu.py."""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=4))
    import __graft_entry__ as ge
    gae = ge.load_package()
    from gae_b200 import ring
    from tests.test_ring_cpu import _oracle_attend, _oracle_merge
    dist.barrier()
    if rank == 1:
        if mode == "leave":
            os._exit(0)  # leaves between steps, nothing in flight
        time.sleep(12)  # "late": misses the exchange by more than the timeout
        os._exit(0)
    q = torch.randn(1, 2, 8, 16)
    t0 = time.time()
    status = "no error"
    try:
        ring.ring_attention(q, q.clone(), q.clone(), causal=True, balance="contiguous",
                            attend=_oracle_attend, merge=_oracle_merge)
    except gae.GAEError as e:
        status = f"{e.status} {time.time() - t0:.1f}"
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(status)
    os._exit(0)


@pytest.mark.parametrize("mode", ["leave", "late"])
def test_ring_reports_a_missing_peer(tmp_path, mode):
    mp.spawn(_worker, args=(2, _port(), mode, str(tmp_path)), nprocs=2, join=True)
    status, secs = (tmp_path / "rank0.txt").read_text().split()
    assert status == "5"          # GAE_ERR_COMM
    assert float(secs) < 11.0     # detected within about the 4 s timeout, no hang


def _bwd_worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=4))
    import __graft_entry__ as ge
    gae = ge.load_package()
    from gae_b200 import ring
    from tests.test_ring_cpu import _block_bwd
    dist.barrier()
    if rank == 1:
        os._exit(0)  # leaves before the backward ring, nothing in flight
    q = torch.randn(1, 2, 8, 16)
    lse = torch.zeros(1, 2, 8)
    t0 = time.time()
    status = "no error"
    try:
        ring.ring_attention_backward(q, q.clone(), q.clone(), q.clone(), q.clone(), lse, causal=True,
                                     balance="contiguous", attend_bwd=_block_bwd)
    except gae.GAEError as e:
        status = f"{e.status} {time.time() - t0:.1f}"
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(status)
    os._exit(0)


def test_ring_backward_reports_a_missing_peer(tmp_path):
    mp.spawn(_bwd_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    status, secs = (tmp_path / "rank0.txt").read_text().split()
    assert status == "5"          # GAE_ERR_COMM
    assert float(secs) < 11.0
