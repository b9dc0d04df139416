/*
 * gae_debug.h -- diagnostics of libgae.so (not part of the attention API).
 *
 * No counterpart in the reference project: these hooks exist to measure the
 * tensor-core attention kernel's pipeline on the GPU.
 */
#ifndef GAE_DEBUG_H_
#define GAE_DEBUG_H_

#include "gae.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Number of events and K/V tiles per event in an attention trace buffer. */
#define GAE_TRACE_EVENTS 12
#define GAE_TRACE_TILES 256

/* Arms (buf != NULL) or disarms (buf == NULL) the cycle-stamp trace of the
 * tensor-core attention kernel on the current device: the CTA with
 * blockIdx = (cta, 0) of every later launch writes %clock64 stamps into
 * buf[event * GAE_TRACE_TILES + tile] (unsigned 64-bit, device memory of
 * GAE_TRACE_EVENTS * GAE_TRACE_TILES entries).  Events: 0/1 softmax group
 * 0/1 saw S, 2/3 group 0/1 published P, 4/5 MMA warp saw P of group 0/1,
 * 6/7 MMA warp issued group 0/1's MMAs for that tile (these per K/V tile
 * of the CTA's first unit); per unit of the CTA: 8 CTA set up (unit 0),
 * 9 group 0 saw the unit's first S, 10/11 group 0 epilogue start / end.  CTA index x counts
 * from the heaviest query block (x = 0 is the last 256 query rows). */
GAE_API gae_status gae_debug_attn_trace(void *buf, int cta);

/* Runs the INT8 attention kernel of gae_attn_int8_fwd (same arguments, same
 * outputs) and has it also write the exact int32 logits q_i . k_j that its
 * softmax threads read back from the tensor memory, logits int32
 * [batch_heads, seq, seq] (tiles wholly above the causal diagonal are not
 * computed and are left as they were).  Pins the bit-exact int32 QK^T of
 * the attention kernel itself (the reference's dot_int8,
 * cuda_src/waller_operator_int8.cu:13-24). */
GAE_API gae_status gae_debug_attn_int8_logits(const gae_attn_int8_args *args, int32_t *logits,
                                              void *stream);

/* The attention launches gae_ring_attn_fwd issues at ring step `step` on
 * `rank` of `world` (shard length shard_len, zigzag != 0 for the balanced
 * causal layout): *n_ops (at most 2) records of 7 int64 in ops: query row 0,
 * query rows, key row 0, key rows (rows of the rank's internal zig-zag or
 * contiguous buffer and of the step's K/V block), causal, absolute position
 * of the first query, of the first key.  Host-only; for tests of the ring's
 * plan without GPUs. */
GAE_API gae_status gae_debug_ring_plan(int rank, int world, int step, int causal, int zigzag,
                                       int64_t shard_len, int64_t *ops, int *n_ops);

/* Exercises the library's bounded device-side wait: launches one thread that
 * waits on an mbarrier nothing will complete, with a limit of timeout_ns
 * (at most 1 s).  The wait gives up, records site 0x901 and the kernel exits
 * normally; gae_device_status() then reports GAE_ERR_TIMEOUT and the CUDA
 * context stays usable.  For testing failure detection without a GPU fault. */
GAE_API gae_status gae_debug_wait_timeout(uint64_t timeout_ns, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* GAE_DEBUG_H_ */
