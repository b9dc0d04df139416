"""Sequence-parallel attention by head/sequence all-to-all ("Ulysses").

An alternative to ring attention for a long sequence whose head count is a
multiple of the GPU count (the reference has no multi-GPU path; this is a new
component).  Every rank holds a contiguous shard [B, H, S, D] of a sequence of
length N = P*S.  One all-to-all turns it into the whole sequence for H/P of
the heads ([B, H/P, N, D]); each rank then runs the library's fused attention
kernel (gae_attn_fwd) over the full sequence of its heads -- one launch, no
per-step merges, and the causal work is identical on every rank -- and a
second all-to-all returns the output to the sequence layout.  Q, K and V
travel as one packed message.

Traffic per rank: 3 tensors in and 1 out, each (P-1)/P of a shard, against
ring attention's P-1 K/V blocks; the compute is one kernel over N.  Remote
data lands in this GPU's memory before any kernel reads it.

`attend` is injectable so that the host logic can run on CPU ranks (gloo) in
tests; the product path uses the CUDA kernel.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist


def _default_attend(q, k, v, causal, scale):
    from . import attention
    return attention(q, k, v, causal=causal, scale=scale)


def _all_to_all(out, inp, group, what):
    try:
        dist.all_to_all_single(out, inp, group=group)
    except Exception as e:  # backend errors carry no common type
        from . import GAEError
        raise GAEError(5, f"ulysses attention: {what} failed: {e}") from e


def ulysses_attention(q, k, v, *, group=None, causal: bool = True, scale: float | None = None,
                      attend=None):
    """Exact attention of this rank's query shard against the whole sequence.

    q, k, v: this rank's contiguous shard [B, H, S, D]; H must be a multiple
    of the number of ranks.  Returns the output shard [B, H, S, D]."""
    attend = attend or _default_attend
    P = dist.get_world_size(group) if dist.is_initialized() else 1
    B, H, S, D = q.shape
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError("ulysses_attention: q, k, v shards must have the same shape")
    if H % P:
        raise ValueError(f"ulysses_attention: heads ({H}) must be a multiple of ranks ({P})")
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    if P == 1:
        return attend(q, k, v, causal, scale)
    Hp = H // P
    # [3, B, H, S, D] -> [P (head group), 3, B, H/P, S, D]: block p goes to rank p.
    packed = torch.stack([q, k, v]).reshape(3, B, P, Hp, S, D).permute(2, 0, 1, 3, 4, 5).contiguous()
    recv = torch.empty_like(packed)  # block p = rank p's sequence shard of my heads
    _all_to_all(recv, packed, group, "gathering the sequence")
    full = recv.permute(1, 2, 3, 0, 4, 5).reshape(3, B, Hp, P * S, D)
    o = attend(full[0], full[1], full[2], causal, scale)  # [B, H/P, N, D], shard p at rows p*S..
    send = o.reshape(B, Hp, P, S, D).permute(2, 0, 1, 3, 4).contiguous()  # block p -> rank p
    back = torch.empty_like(send)  # block p = head group p of my sequence shard
    _all_to_all(back, send, group, "returning the output")
    return back.permute(1, 0, 2, 3, 4).reshape(B, H, S, D)
