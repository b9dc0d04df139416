"""Sequence-parallel exact causal attention over P GPUs (ring attention).

A new component (the reference has no multi-GPU path): one process per GPU,
torch.distributed over NCCL for the plumbing, the library's fused attention
kernel (gae_attn_fwd with q_offset/kv_offset) for each block pair and its
log-sum-exp merge kernel (gae_lse_merge) to combine partial results, the same
algebra as the reference's (max, sum, acc) block merge
(cuda_src/waller_operator_v2.cu:120-142).

Layout.  Every rank holds a contiguous shard [B, H, S, D] of a sequence of
length N = P*S (rank r owns positions [r*S, (r+1)*S)).  With
balance="zigzag" (the default for causal attention) the shards are first
re-dealt so that rank r owns chunks r and 2P-1-r of 2P equal chunks; every
ring step then costs every rank the same two chunk-pairs of work, instead of
rank r doing r+1/2 blocks of work under the contiguous layout.  The output is
dealt back to the contiguous layout at the end.

Ring step t (t = 0 .. P-1): rank r computes with the K/V of rank (r - t) mod P
while it sends that block to rank r+1 and receives the next one from rank r-1
(batch_isend_irecv on NCCL's stream, overlapped with the attention kernels on
the compute stream).  K and V travel as one packed buffer; remote blocks land
in this GPU's own memory before any kernel reads them.

Failure handling: a rank that dies, leaves, or never joins a step makes the
other ranks' exchange fail (an error from the backend or the process group's
timeout); the driver raises GAEError(GAE_ERR_COMM) naming the step.  The
timeout is the process group's (init_process_group(timeout=...)).

Two host paths with one algorithm.  On CUDA tensors with no injected
`attend`/`merge`, ring_attention is a thin caller of the library's C ABI
(gae_ring_ctx_create / gae_ring_attn_fwd): the re-deal, the K/V rotation
over NCCL send/recv, the attention launches and the merges run in libgae.so
(one communicator per process group, created on first use from a unique id
broadcast over the group).  With `attend` and `merge` injected (CPU gloo
tests), the same plan runs here in Python over torch.distributed.  The
product path fails loudly without the CUDA library.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist


def _default_attend(q, k, v, causal, q_offset, kv_offset, scale):
    from . import attention
    return attention(q, k, v, causal=causal, q_offset=q_offset, kv_offset=kv_offset,
                     scale=scale, return_lse=True)


def _default_merge(o_acc, lse_acc, o_part, lse_part):
    from . import lse_merge_
    lse_merge_(o_acc, lse_acc, o_part, lse_part)


def _comm_error(what, exc):
    from . import GAEError
    return GAEError(5, f"ring attention: {what} failed: {exc}")


def _exchange(ops, what):
    """Runs a batch of point-to-point operations and waits for it.  A peer
    that died, left, or stayed away past the process group's timeout surfaces
    here as GAEError(GAE_ERR_COMM) instead of an opaque backend error."""
    try:
        for w in dist.batch_isend_irecv(ops):
            w.wait()
    except Exception as e:  # backend errors carry no common type
        raise _comm_error(what, e) from e


def zigzag_owner(chunk: int, P: int) -> int:
    """Rank that owns chunk `chunk` (of 2P) under the balanced layout."""
    return chunk if chunk < P else 2 * P - 1 - chunk


def _redeal(x, rank, P, group, to_zigzag: bool):
    """Moves the two half-shards between the contiguous and zig-zag layouts.

    Contiguous rank r holds chunks 2r, 2r+1; zig-zag rank r holds chunks
    r, 2P-1-r.  Point-to-point exchange, 2 sends and 2 receives per rank."""
    S = x.shape[2]
    C = S // 2
    out = torch.empty_like(x)
    ops, local = [], []
    if to_zigzag:
        # send my contiguous chunks to their zig-zag owners
        for i, ch in enumerate((2 * rank, 2 * rank + 1)):
            dst = zigzag_owner(ch, P)
            slot = 0 if ch < P else 1
            src_view = x[:, :, i * C:(i + 1) * C].contiguous()
            if dst == rank:
                local.append((out[:, :, slot * C:(slot + 1) * C], src_view))
            else:
                ops.append(dist.P2POp(dist.isend, src_view, dst, group))
        # receive my zig-zag chunks from their contiguous owners
        recv = []
        for slot, ch in enumerate((rank, 2 * P - 1 - rank)):
            src = ch // 2
            if src != rank:
                buf = torch.empty_like(x[:, :, :C])
                ops.append(dist.P2POp(dist.irecv, buf, src, group))
                recv.append((out[:, :, slot * C:(slot + 1) * C], buf))
    else:
        for slot, ch in enumerate((rank, 2 * P - 1 - rank)):
            dst = ch // 2
            i = ch % 2
            src_view = x[:, :, slot * C:(slot + 1) * C].contiguous()
            if dst == rank:
                local.append((out[:, :, i * C:(i + 1) * C], src_view))
            else:
                ops.append(dist.P2POp(dist.isend, src_view, dst, group))
        recv = []
        for i, ch in enumerate((2 * rank, 2 * rank + 1)):
            src = zigzag_owner(ch, P)
            if src != rank:
                buf = torch.empty_like(x[:, :, :C])
                ops.append(dist.P2POp(dist.irecv, buf, src, group))
                recv.append((out[:, :, i * C:(i + 1) * C], buf))
    for dst_view, src_view in local:
        dst_view.copy_(src_view)
    if ops:
        _exchange(ops, "re-dealing the shards")
    for dst_view, buf in recv:
        dst_view.copy_(buf)
    return out


_CTX = {}
RING_TIMEOUT_S = 120.0  # bound on every wait of the C-ABI ring (communicator and completion)


def _group_key(group):
    return (None if group is None else id(group), __import__("torch").cuda.current_device())


def ring_context(group=None, timeout_s: float = RING_TIMEOUT_S):
    """The C-ABI ring context of `group` on the current device (created on
    first use, collectively: rank 0 of the group makes an NCCL unique id and
    broadcasts it over the group)."""
    import ctypes as C
    from . import lib, _check
    key = _group_key(group)
    if key in _CTX:
        return _CTX[key]
    P = dist.get_world_size(group) if dist.is_initialized() else 1
    r = dist.get_rank(group) if dist.is_initialized() else 0
    uid = (C.c_ubyte * 128)()
    if r == 0 and P > 1:  # one rank needs no communicator
        _check(lib().gae_ring_unique_id(uid))
    if P > 1:
        obj = [bytes(uid)]
        src = dist.get_global_rank(group, 0) if group is not None else 0
        try:
            dist.broadcast_object_list(obj, src=src, group=group)
        except Exception as e:
            raise _comm_error("sharing the ring's NCCL id", e) from e
        C.memmove(uid, obj[0], 128)
    ctx = C.c_void_p()
    _check(lib().gae_ring_ctx_create(uid, r, P, float(timeout_s), C.byref(ctx)))
    _CTX[key] = ctx
    return ctx


def release_contexts():
    """Destroys every C-ABI ring context of this process (collective over
    each context's ranks)."""
    from . import lib
    for key in list(_CTX):
        lib().gae_ring_ctx_destroy(_CTX.pop(key))


def _ring_attention_native(q, k, v, group, causal, balance, scale, return_lse):
    import ctypes as C
    from . import lib, _check, _attn_args, _stream_ptr
    B, H, S, D = q.shape
    out = torch.empty_like(q)
    lse = torch.empty((B, H, S), dtype=torch.float32, device=q.device) if return_lse else None
    a = _attn_args(q, k, v, out, lse, causal, scale)
    bal = 0 if balance == "zigzag" else 1
    _check(lib().gae_ring_attn_fwd(ring_context(group), C.byref(a), bal, _stream_ptr(None)))
    return (out, lse) if return_lse else out


def ring_attention(q, k, v, *, group=None, causal: bool = True, balance: str = "zigzag",
                   scale: float | None = None, return_lse: bool = False, attend=None,
                   merge=None):
    """Exact attention of this rank's query shard against the whole sequence.

    q, k, v: this rank's contiguous shard [B, H, S, D].  Returns the output
    shard (dtype of q) and, with return_lse, the fp32 log-sum-exp [B, H, S].
    """
    if balance not in ("zigzag", "contiguous"):
        raise ValueError(f"unknown balance {balance!r}")
    if attend is None and merge is None and q.is_cuda:
        if k.shape != q.shape or v.shape != q.shape:
            raise ValueError("ring_attention: q, k, v shards must have the same shape")
        if causal and balance == "zigzag" and q.shape[2] % 2 and \
                (dist.get_world_size(group) if dist.is_initialized() else 1) > 1:
            raise ValueError("ring_attention: zig-zag balance needs an even shard length")
        return _ring_attention_native(q, k, v, group, causal, balance, scale, return_lse)
    attend = attend or _default_attend
    merge = merge or _default_merge
    P = dist.get_world_size(group) if dist.is_initialized() else 1
    r = dist.get_rank(group) if dist.is_initialized() else 0
    B, H, S, D = q.shape
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError("ring_attention: q, k, v shards must have the same shape")
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    zig = causal and balance == "zigzag"
    if zig and S % 2:
        raise ValueError("ring_attention: zig-zag balance needs an even shard length")
    if balance not in ("zigzag", "contiguous"):
        raise ValueError(f"unknown balance {balance!r}")

    # Local chunks: (global chunk id, offset in the local buffer, length).
    if zig:
        C = S // 2
        q, k, v = (_redeal(t, r, P, group, True) if P > 1 else t for t in (q, k, v))
        chunks_of = lambda rank: [(rank, 0, C), (2 * P - 1 - rank, C, C)]
    else:
        C = S
        chunks_of = lambda rank: [(rank, 0, S)]

    kv = torch.stack([k, v])  # one packed message per step
    kv_next = torch.empty_like(kv) if P > 1 else None
    acc = [None] * len(chunks_of(r))  # per local q chunk: (o fp32, lse)

    for t in range(P):
        src = (r - t) % P
        reqs = []
        if t < P - 1:
            ops = [dist.P2POp(dist.isend, kv, (r + 1) % P, group),
                   dist.P2POp(dist.irecv, kv_next, (r - 1) % P, group)]
            try:
                reqs = dist.batch_isend_irecv(ops)
            except Exception as e:
                raise _comm_error(f"posting the K/V exchange of step {t}", e) from e
        for qi, (qc, qo, ql) in enumerate(chunks_of(r)):
            for kc, ko, kl in chunks_of(src):
                if causal and kc > qc:
                    continue  # every key after every query: fully masked
                diag = causal and kc == qc
                o_p, l_p = attend(q[:, :, qo:qo + ql], kv[0][:, :, ko:ko + kl],
                                  kv[1][:, :, ko:ko + kl], diag, qc * C, kc * C, scale)
                if acc[qi] is None:
                    acc[qi] = (o_p.float().contiguous(), l_p.contiguous())
                else:
                    merge(acc[qi][0], acc[qi][1], o_p.contiguous(), l_p.contiguous())
        try:
            for w in reqs:
                w.wait()
        except Exception as e:
            raise _comm_error(f"the K/V exchange of step {t}", e) from e
        if t < P - 1:
            kv, kv_next = kv_next, kv

    out = torch.empty_like(q)
    lse = torch.empty((B, H, S), dtype=torch.float32, device=q.device)
    for (qc, qo, ql), a in zip(chunks_of(r), acc):
        out[:, :, qo:qo + ql] = a[0].to(out.dtype)
        lse[:, :, qo:qo + ql] = a[1]
    if zig and P > 1:
        out = _redeal(out, r, P, group, False)
        lse = _redeal(lse.unsqueeze(-1), r, P, group, False).squeeze(-1)
    return (out, lse) if return_lse else out


def _default_attend_bwd(q, k, v, out, dout, lse, causal, scale):
    from . import attention_backward
    return attention_backward(q, k, v, out, dout, lse, causal=causal, scale=scale)


def ring_attention_backward(q, k, v, out, dout, lse, *, group=None, causal: bool = True,
                            balance: str = "zigzag", scale: float | None = None, attend_bwd=None):
    """Gradients (dq, dk, dv) of ring_attention for this rank's shards.

    q, k, v, dout: this rank's contiguous shards [B, H, S, D]; out and lse:
    this rank's output and log-sum-exp from ring_attention(return_lse=True)
    with the same group, causal and balance.  Each block pair goes through
    the library's backward kernel (gae_attn_bwd) with the final output and
    LSE of the query rows, which makes the per-pair gradients exact parts of
    the full ones: dq sums over the K/V blocks this rank meets, and each K/V
    block carries fp32 dK/dV accumulators around the ring with it, handed on
    after every step and returned to the block's owner after the last one.
    """
    attend_bwd = attend_bwd or _default_attend_bwd
    P = dist.get_world_size(group) if dist.is_initialized() else 1
    r = dist.get_rank(group) if dist.is_initialized() else 0
    B, H, S, D = q.shape
    for t in (k, v, out, dout):
        if t.shape != q.shape:
            raise ValueError("ring_attention_backward: q, k, v, out, dout shards must have the same shape")
    if lse.shape != (B, H, S):
        raise ValueError("ring_attention_backward: lse must be [B, H, S]")
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    zig = causal and balance == "zigzag"
    if zig and S % 2:
        raise ValueError("ring_attention_backward: zig-zag balance needs an even shard length")
    if balance not in ("zigzag", "contiguous"):
        raise ValueError(f"unknown balance {balance!r}")

    if zig:
        C = S // 2
        if P > 1:
            q, k, v, out, dout = (_redeal(t, r, P, group, True) for t in (q, k, v, out, dout))
            lse = _redeal(lse.unsqueeze(-1), r, P, group, True).squeeze(-1)
        chunks_of = lambda rank: [(rank, 0, C), (2 * P - 1 - rank, C, C)]
    else:
        C = S
        chunks_of = lambda rank: [(rank, 0, S)]

    kv = torch.stack([k, v])
    kv_next = torch.empty_like(kv) if P > 1 else None
    dkv = torch.zeros(kv.shape, dtype=torch.float32, device=q.device)  # travels with kv
    dkv_next = torch.empty_like(dkv) if P > 1 else None
    dq = torch.zeros(q.shape, dtype=torch.float32, device=q.device)

    for t in range(P):
        src = (r - t) % P
        reqs = []
        if t < P - 1:  # the next K/V block travels while this one is used
            try:
                reqs = dist.batch_isend_irecv([dist.P2POp(dist.isend, kv, (r + 1) % P, group),
                                               dist.P2POp(dist.irecv, kv_next, (r - 1) % P, group)])
            except Exception as e:
                raise _comm_error(f"posting the K/V exchange of backward step {t}", e) from e
        for qc, qo, ql in chunks_of(r):
            qs = slice(qo, qo + ql)
            lse_c = lse[:, :, qs].contiguous()
            for kc, ko, kl in chunks_of(src):
                if causal and kc > qc:
                    continue  # every key after every query: no gradient
                ks = slice(ko, ko + kl)
                dq_p, dk_p, dv_p = attend_bwd(q[:, :, qs], kv[0][:, :, ks], kv[1][:, :, ks],
                                              out[:, :, qs], dout[:, :, qs], lse_c,
                                              causal and kc == qc, scale)
                dq[:, :, qs] += dq_p.float()
                dkv[0][:, :, ks] += dk_p.float()
                dkv[1][:, :, ks] += dv_p.float()
        try:
            for w in reqs:
                w.wait()
        except Exception as e:
            raise _comm_error(f"the K/V exchange of backward step {t}", e) from e
        if P > 1:
            # Hand this block's accumulators on with it (after the last step
            # they reach the block's owner).
            _exchange([dist.P2POp(dist.isend, dkv, (r + 1) % P, group),
                       dist.P2POp(dist.irecv, dkv_next, (r - 1) % P, group)],
                      f"the dK/dV exchange of backward step {t}")
            dkv, dkv_next = dkv_next, dkv
            if t < P - 1:
                kv, kv_next = kv_next, kv

    dq, dk, dv = dq.to(q.dtype), dkv[0].to(q.dtype), dkv[1].to(q.dtype)
    if zig and P > 1:
        dq, dk, dv = (_redeal(t, r, P, group, False) for t in (dq, dk, dv))
    return dq, dk, dv
