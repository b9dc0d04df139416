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


def _default_attend(q, k, v, causal, scale, return_lse=False):
    from . import attention
    return attention(q, k, v, causal=causal, scale=scale, return_lse=return_lse)


def _default_attend_bwd(q, k, v, out, dout, lse, causal, scale):
    from . import attention_backward
    return attention_backward(q, k, v, out, dout, lse, causal=causal, scale=scale)


def _all_to_all(out, inp, group, what):
    try:
        dist.all_to_all_single(out, inp, group=group)
    except Exception as e:  # backend errors carry no common type
        from . import GAEError
        raise GAEError(5, f"ulysses attention: {what} failed: {e}") from e


def _to_heads(ts, P, group, what):
    """Sequence shards [B, H, S, D] (one packed message) -> the whole sequence
    for this rank's H/P heads, [B, H/P, P*S, D] each."""
    n = len(ts)
    B, H, S, D = ts[0].shape
    Hp = H // P
    # [n, B, H, S, D] -> [P (head group), n, B, H/P, S, D]: block p goes to rank p.
    packed = torch.stack(ts).reshape(n, B, P, Hp, S, D).permute(2, 0, 1, 3, 4, 5).contiguous()
    recv = torch.empty_like(packed)  # block p = rank p's sequence shard of my heads
    _all_to_all(recv, packed, group, what)
    full = recv.permute(1, 2, 3, 0, 4, 5).reshape(n, B, Hp, P * S, D)
    return [full[i] for i in range(n)]


def _to_seq(ts, P, group, what):
    """Inverse of _to_heads: [B, H/P, P*S, D] -> this rank's shard [B, H, S, D]."""
    n = len(ts)
    B, Hp, N, D = ts[0].shape
    S = N // P
    send = torch.stack(ts).reshape(n, B, Hp, P, S, D).permute(3, 0, 1, 2, 4, 5).contiguous()
    back = torch.empty_like(send)  # block p = head group p of my sequence shard
    _all_to_all(back, send, group, what)
    return [back[:, i].permute(1, 0, 2, 3, 4).reshape(B, P * Hp, S, D) for i in range(n)]


def _check(q, others, P, name):
    B, H, S, D = q.shape
    for t in others:
        if t.shape != q.shape:
            raise ValueError(f"{name}: shards must have the same shape")
    if H % P:
        raise ValueError(f"{name}: heads ({H}) must be a multiple of ranks ({P})")


def ulysses_attention(q, k, v, *, group=None, causal: bool = True, scale: float | None = None,
                      attend=None, return_lse: bool = False):
    """Exact attention of this rank's query shard against the whole sequence.

    q, k, v: this rank's contiguous shard [B, H, S, D]; H must be a multiple
    of the number of ranks.  Returns the output shard [B, H, S, D] and, with
    return_lse, its fp32 log-sum-exp [B, H, S] (attend then returns (o, lse))."""
    attend = attend or _default_attend
    P = dist.get_world_size(group) if dist.is_initialized() else 1
    _check(q, (k, v), P, "ulysses_attention")
    D = q.shape[-1]
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    if P == 1:
        return attend(q, k, v, causal, scale, True) if return_lse else attend(q, k, v, causal, scale)
    fq, fk, fv = _to_heads([q, k, v], P, group, "gathering the sequence")
    res = attend(fq, fk, fv, causal, scale, True) if return_lse else attend(fq, fk, fv, causal, scale)
    o, lse = res if return_lse else (res, None)
    (out,) = _to_seq([o], P, group, "returning the output")
    if not return_lse:
        return out
    (l,) = _to_seq([lse.unsqueeze(-1)], P, group, "returning the log-sum-exp")
    return out, l.squeeze(-1).contiguous()


def ulysses_attention_backward(q, k, v, out, dout, lse, *, group=None, causal: bool = True,
                               scale: float | None = None, attend_bwd=None):
    """Gradients (dq, dk, dv) of ulysses_attention for this rank's shards:
    q, k, v, out, dout [B, H, S, D] and lse [B, H, S] from
    ulysses_attention(return_lse=True).  One all-to-all gathers the sequence
    for H/P heads, one backward launch (gae_attn_bwd) runs over it, and a
    second all-to-all returns the gradients to the sequence layout."""
    attend_bwd = attend_bwd or _default_attend_bwd
    P = dist.get_world_size(group) if dist.is_initialized() else 1
    _check(q, (k, v, out, dout), P, "ulysses_attention_backward")
    D = q.shape[-1]
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    if P == 1:
        return attend_bwd(q, k, v, out, dout, lse, causal, scale)
    fq, fk, fv, fo, fd = _to_heads([q, k, v, out, dout], P, group, "gathering the sequence")
    (fl,) = _to_heads([lse.unsqueeze(-1)], P, group, "gathering the log-sum-exp")
    dq, dk, dv = attend_bwd(fq, fk, fv, fo, fd, fl.squeeze(-1).contiguous(), causal, scale)
    return tuple(_to_seq([dq, dk, dv], P, group, "returning the gradients"))
