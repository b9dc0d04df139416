// ring.cuh -- sequence-parallel ring attention behind the C ABI
// (gae_ring_ctx_create / gae_ring_attn_fwd / gae_ring_ctx_destroy).
//
// A new component: the reference has no multi-GPU path.  One process (or
// thread) per GPU; this rank holds a contiguous shard [B, H, S, D] of one
// sequence of N = P*S tokens.  With zig-zag balance (causal) the shards are
// first re-dealt so that rank r holds chunks r and 2P-1-r of 2P equal chunks
// (every ring step then costs every rank the same work); per ring step t the
// rank attends its queries to the K/V block of rank (r - t) mod P while NCCL
// moves that block on to rank r+1 and brings the next one from rank r-1 (on
// a communication stream, overlapped with the attention launches on the
// caller's stream).  Partial outputs are merged by log-sum-exp into an fp32
// accumulator; the result is dealt back to the contiguous layout.  Remote
// blocks always land in this GPU's memory before a kernel reads them (no peer
// loads, no TMA multicast).
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, preferring a copy the
// process already loaded), so the library has no link-time NCCL dependency
// and its other entry points work without it.  The communicator is
// non-blocking; every wait on it is bounded by the context's timeout, after
// which the communicator is aborted and the call returns GAE_ERR_TIMEOUT
// (GAE_ERR_COMM for an error NCCL reports).
//
// This header is included by gae_abi.cu after its helpers (fail, the
// attention launcher): one translation unit.
#pragma once
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <thread>

namespace gae {

// ---------------------------------------------------------------- kernels
// dst[b, h, s, :] = src[b, h, s, :] for s < rows over [B, H, rows, D] views
// with element strides {b, h, s} on both sides (head_dim contiguous); the
// element types may differ (fp32 accumulator -> 16-bit output).  One warp a
// row; vec4: D, every stride and both bases allow 4-element vector accesses.
template <typename TS, typename TD>
__global__ void ring_copy_rows_kernel(const TS *__restrict__ src, int64_t ssb, int64_t ssh, int64_t sss,
                                      TD *__restrict__ dst, int64_t dsb, int64_t dsh, int64_t dss,
                                      int H, int64_t rows, int64_t total_rows, int D, int vec4) {
    const int64_t g = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (g >= total_rows) return;
    const int lane = threadIdx.x & 31;
    const int64_t s = g % rows, bh = g / rows;
    const int64_t b = bh / H, h = bh % H;
    const TS *sr = src + b * ssb + h * ssh + s * sss;
    TD *dr = dst + b * dsb + h * dsh + s * dss;
    if (vec4) {  // four elements a lane, one vector load and store each
        for (int c = 4 * lane; c < D; c += 128) {
            float f[4];
            if constexpr (sizeof(TS) == 4) {
                const float4 x = *reinterpret_cast<const float4 *>(sr + c);
                f[0] = x.x; f[1] = x.y; f[2] = x.z; f[3] = x.w;
            } else {
                const uint2 x = *reinterpret_cast<const uint2 *>(sr + c);
                const TS *e = reinterpret_cast<const TS *>(&x);
#pragma unroll
                for (int u = 0; u < 4; ++u) f[u] = to_f<TS>(e[u]);
            }
            if constexpr (sizeof(TD) == 4) {
                *reinterpret_cast<float4 *>(dr + c) = make_float4(f[0], f[1], f[2], f[3]);
            } else {
                uint2 y;
                TD *e = reinterpret_cast<TD *>(&y);
#pragma unroll
                for (int u = 0; u < 4; ++u) e[u] = from_f<TD>(f[u]);
                *reinterpret_cast<uint2 *>(dr + c) = y;
            }
        }
        return;
    }
    for (int c = lane; c < D; c += 32) dr[c] = from_f<TD>(to_f<TS>(sr[c]));
}

// lse_acc[bh, row0 + i] and acc[bh, row0 + i, :] (fp32, dense [BH, acc_rows,
// D]) absorb a partial result over other keys: part [BH, rows, D] (16-bit,
// dense) with lse_part [BH, rows]; the (max, sum) merge in log-sum-exp form.
template <typename TP>
__global__ void ring_merge_kernel(float *__restrict__ acc, float *__restrict__ lse_acc,
                                  const TP *__restrict__ part, const float *__restrict__ lse_part,
                                  int64_t rows, int64_t acc_rows, int64_t row0, int64_t total_rows, int D) {
    const int64_t g = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (g >= total_rows) return;
    const int lane = threadIdx.x & 31;
    const int64_t i = g % rows, bh = g / rows;
    const int64_t ra = bh * acc_rows + row0 + i;
    const float la = lse_acc[ra], lb = lse_part[g];
    const float mx = fmaxf(la, lb);
    if (mx == -INFINITY) return;
    const float wa = expf(la - mx), wb = expf(lb - mx);
    const float s = wa + wb;
    float *oa = acc + ra * D;
    const TP *op = part + g * D;
    for (int c = lane; c < D; c += 32) oa[c] = (wa * oa[c] + wb * to_f<TP>(op[c])) / s;
    __syncwarp();
    if (lane == 0) lse_acc[ra] = mx + logf(s);
}

__global__ void ring_fill_kernel(float *__restrict__ x, int64_t n, float v) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = v;
}

}  // namespace gae

namespace {

// ------------------------------------------------------------ ring plan
// One attention launch of a ring step, in rows of this rank's zig-zag (or
// contiguous) buffer: queries [q_row0, q_row0 + q_rows) against keys
// [kv_row0, kv_row0 + kv_rows) of the step's K/V block, with absolute
// positions q_pos / kv_pos of the first row / key (used only when causal);
// the partial result is merged into accumulator rows starting at q_row0.
struct RingOp {
    int step;
    int64_t q_row0, q_rows, kv_row0, kv_rows;
    int causal;
    int64_t q_pos, kv_pos;
};

// The launches of ring step t on rank r (world P, shard length S).  zig:
// chunks (r, 2P-1-r) of length C = S/2 in rows [0, C), [C, 2C).  Adjacent
// chunks are covered by one launch wherever their masks allow:
//   t = 0: q chunk 0 vs k chunk 0 (diagonal), q chunk 1 vs k chunks 0-1
//          (chunk 0's keys all precede chunk 1's queries, so treating them
//          as the C positions just before chunk 1 gives the same mask);
//   src < r: both q chunks vs k chunk 0 (all visible);
//   src > r: q chunk 1 vs both k chunks (all visible).
// Contiguous layout: the whole shard vs the block, causal only on the
// diagonal, skipped above it.
int ring_plan(int r, int P, int t, int causal, int zig, int64_t S, RingOp *ops) {
    const int src = ((r - t) % P + P) % P;
    int n = 0;
    if (zig) {
        const int64_t C = S / 2;
        if (t == 0) {
            ops[n++] = RingOp{t, 0, C, 0, C, 1, (int64_t)r * C, (int64_t)r * C};
            ops[n++] = RingOp{t, C, C, 0, 2 * C, 1, (int64_t)(2 * P - 1 - r) * C, (int64_t)(2 * P - 2 - r) * C};
        } else if (src < r) {
            ops[n++] = RingOp{t, 0, 2 * C, 0, C, 0, 0, 0};
        } else {
            ops[n++] = RingOp{t, C, C, 0, 2 * C, 0, 0, 0};
        }
        return n;
    }
    if (!causal) {
        ops[n++] = RingOp{t, 0, S, 0, S, 0, 0, 0};
    } else if (src == r) {
        ops[n++] = RingOp{t, 0, S, 0, S, 1, (int64_t)r * S, (int64_t)r * S};
    } else if (src < r) {
        ops[n++] = RingOp{t, 0, S, 0, S, 0, 0, 0};
    }
    return n;
}

// ------------------------------------------------------------ NCCL loader
struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId *);
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*CommFinalize)(ncclComm_t);
    ncclResult_t (*CommCount)(const ncclComm_t, int *);
    ncclResult_t (*CommUserRank)(const ncclComm_t, int *);
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    const char *(*GetErrorString)(ncclResult_t);
    bool ok;
};

const NcclApi *nccl_api() {
    static NcclApi api = [] {
        NcclApi a;
        memset(&a, 0, sizeof(a));
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the process's copy first
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return a;
#define GAE_NCCL_SYM(field, name)                                  \
    a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, name)); \
    if (!a.field) return a;
        GAE_NCCL_SYM(GetUniqueId, "ncclGetUniqueId");
        GAE_NCCL_SYM(CommInitRankConfig, "ncclCommInitRankConfig");
        GAE_NCCL_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
        GAE_NCCL_SYM(CommAbort, "ncclCommAbort");
        GAE_NCCL_SYM(CommDestroy, "ncclCommDestroy");
        GAE_NCCL_SYM(CommFinalize, "ncclCommFinalize");
        GAE_NCCL_SYM(CommCount, "ncclCommCount");
        GAE_NCCL_SYM(CommUserRank, "ncclCommUserRank");
        GAE_NCCL_SYM(Send, "ncclSend");
        GAE_NCCL_SYM(Recv, "ncclRecv");
        GAE_NCCL_SYM(GroupStart, "ncclGroupStart");
        GAE_NCCL_SYM(GroupEnd, "ncclGroupEnd");
        GAE_NCCL_SYM(GetErrorString, "ncclGetErrorString");
#undef GAE_NCCL_SYM
        a.ok = true;
        return a;
    }();
    return api.ok ? &api : nullptr;
}

}  // namespace

// ------------------------------------------------------------ ring context
struct gae_ring_ctx {
    const NcclApi *nc = nullptr;
    ncclComm_t comm = nullptr;
    bool owns_comm = false;
    bool dead = false;  // aborted after a failure: every later call fails
    int rank = 0, world = 1, device = 0;
    double timeout_s = 0.0;
    cudaStream_t comm_st = nullptr;
    cudaEvent_t ev_a = nullptr, ev_b = nullptr, ev_done = nullptr;
    void *buf = nullptr;  // one device arena, grown on demand
    size_t buf_bytes = 0;
};

namespace {

using Clock = std::chrono::steady_clock;

double secs_since(Clock::time_point t0) {
    return std::chrono::duration<double>(Clock::now() - t0).count();
}

// Marks the context dead after aborting its communicator (which also
// releases NCCL kernels that wait on a peer).
gae_status ring_fail(gae_ring_ctx *c, gae_status s, const char *what, const char *detail) {
    if (c->comm && c->owns_comm && !c->dead) c->nc->CommAbort(c->comm);
    c->dead = true;
    return fail(s, "ring attention: %s: %s", what, detail);
}

// Waits until a non-blocking NCCL call has taken effect (bounded).
gae_status nccl_settle(gae_ring_ctx *c, ncclResult_t r, const char *what) {
    const auto t0 = Clock::now();
    while (r == ncclInProgress) {
        if (c->timeout_s > 0 && secs_since(t0) > c->timeout_s)
            return ring_fail(c, GAE_ERR_TIMEOUT, what, "NCCL call did not complete within the timeout");
        std::this_thread::yield();
        ncclResult_t st = ncclSuccess;
        if (c->nc->CommGetAsyncError(c->comm, &st) != ncclSuccess) st = ncclSystemError;
        r = st;
    }
    if (r != ncclSuccess) return ring_fail(c, GAE_ERR_COMM, what, c->nc->GetErrorString(r));
    return GAE_OK;
}

// Waits for `ev` (bounded), watching the communicator for errors.
gae_status ring_wait_event(gae_ring_ctx *c, cudaEvent_t ev, const char *what) {
    const auto t0 = Clock::now();
    for (;;) {
        const cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return GAE_OK;
        if (e != cudaErrorNotReady) return ring_fail(c, GAE_ERR_CUDA, what, cudaGetErrorString(e));
        ncclResult_t st = ncclSuccess;
        if (c->nc->CommGetAsyncError(c->comm, &st) != ncclSuccess || (st != ncclSuccess && st != ncclInProgress))
            return ring_fail(c, GAE_ERR_COMM, what, c->nc->GetErrorString(st));
        if (c->timeout_s > 0 && secs_since(t0) > c->timeout_s)
            return ring_fail(c, GAE_ERR_TIMEOUT, what, "no completion within the timeout");
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

gae_status ring_ctx_init_common(gae_ring_ctx *c) {
    GAE_CUDA_TRY(cudaGetDevice(&c->device));
    GAE_CUDA_TRY(cudaStreamCreateWithFlags(&c->comm_st, cudaStreamNonBlocking));
    GAE_CUDA_TRY(cudaEventCreateWithFlags(&c->ev_a, cudaEventDisableTiming));
    GAE_CUDA_TRY(cudaEventCreateWithFlags(&c->ev_b, cudaEventDisableTiming));
    GAE_CUDA_TRY(cudaEventCreateWithFlags(&c->ev_done, cudaEventDisableTiming));
    return GAE_OK;
}

void ring_ctx_release(gae_ring_ctx *c) {
    if (c->comm_st) cudaStreamSynchronize(c->comm_st);
    if (c->buf) cudaFree(c->buf);
    if (c->ev_a) cudaEventDestroy(c->ev_a);
    if (c->ev_b) cudaEventDestroy(c->ev_b);
    if (c->ev_done) cudaEventDestroy(c->ev_done);
    if (c->comm_st) cudaStreamDestroy(c->comm_st);
    if (c->comm && c->owns_comm) {
        if (!c->dead && nccl_settle(c, c->nc->CommFinalize(c->comm), "finalising the communicator") == GAE_OK)
            c->nc->CommDestroy(c->comm);
        else if (!c->dead)
            c->nc->CommAbort(c->comm);
    }
    delete c;
}

gae_status ring_reserve(gae_ring_ctx *c, size_t bytes) {
    if (bytes <= c->buf_bytes) return GAE_OK;
    if (c->buf) {
        GAE_CUDA_TRY(cudaDeviceSynchronize());  // earlier calls may still use it
        GAE_CUDA_TRY(cudaFree(c->buf));
        c->buf = nullptr;
        c->buf_bytes = 0;
    }
    GAE_CUDA_TRY(cudaMalloc(&c->buf, bytes));
    c->buf_bytes = bytes;
    return GAE_OK;
}

template <typename TS, typename TD>
gae_status ring_copy(const TS *src, const int64_t ss[3], TD *dst, const int64_t ds[3], int64_t B, int64_t H,
                     int64_t rows, int64_t D, cudaStream_t st) {
    const int64_t total = B * H * rows;
    if (total == 0) return GAE_OK;
    const int warps = 8;
    auto al = [](const void *p, size_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; };
    const int vec4 = (D % 4 == 0) && al(src, 4 * sizeof(TS)) && al(dst, 4 * sizeof(TD)) && ss[0] % 4 == 0 &&
                     ss[1] % 4 == 0 && ss[2] % 4 == 0 && ds[0] % 4 == 0 && ds[1] % 4 == 0 && ds[2] % 4 == 0;
    gae::ring_copy_rows_kernel<TS, TD><<<(unsigned)((total + warps - 1) / warps), warps * 32, 0, st>>>(
        src, ss[0], ss[1], ss[2], dst, ds[0], ds[1], ds[2], (int)H, rows, total, (int)D, vec4);
    GAE_CUDA_TRY(cudaGetLastError());
    return GAE_OK;
}

// Diagnostics: GAE_RING_PROFILE=1 prints each phase's device time (CUDA
// events on the two streams) to stderr after every call.  Off by default.
struct RingProfile {
    bool on = false;
    cudaEvent_t ev[64];
    cudaStream_t evs[64];
    const char *name[64];
    int n = 0;
    explicit RingProfile(bool enable) : on(enable) {}
    void mark(const char *what, cudaStream_t stream) {
        if (!on || n >= 64) return;
        cudaEventCreate(&ev[n]);
        cudaEventRecord(ev[n], stream);
        evs[n] = stream;
        name[n++] = what;
    }
    void report(int rank) {
        if (!on) return;
        for (int i = 0; i < n; ++i) cudaEventSynchronize(ev[i]);
        for (int i = 1; i < n; ++i) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, ev[0], ev[i]);
            fprintf(stderr, "[gae ring rank %d] %-24s at %9.3f ms\n", rank, name[i], ms);
        }
        for (int i = 0; i < n; ++i) cudaEventDestroy(ev[i]);
        n = 0;
    }
};

template <typename T>
gae_status ring_run(gae_ring_ctx *c, const gae_attn_args *a, int zig, cudaStream_t st) {
    static const bool prof_on = [] {
        const char *e = getenv("GAE_RING_PROFILE");
        return e && e[0] == '1';
    }();
    RingProfile prof(prof_on);
    prof.mark("start", st);
    const int P = c->world, r = c->rank;
    const int64_t B = a->batch, H = a->heads, S = a->seq_q, D = a->head_dim, BH = B * H;
    const int64_t C = zig ? S / 2 : S;
    const size_t es = sizeof(T);
    const ncclDataType_t nt = ncclUint8;  // bytes on the wire
    // Arena: zq [BH, S, D] | kv[2] [2, BH, S, D] | acc fp32 [BH, S, D] |
    // lse_acc [BH, S] | part [BH, S, D] | lse_part [BH, S] | re-deal staging:
    // send [2 chunks][q|k|v][BH, C, D] and receive [2 chunks][q|k|v][BH, C, D]
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    const size_t act = (size_t)BH * S * D;
    size_t off = 0;
    const size_t o_zq = off; off += al(act * es);
    const size_t o_kv0 = off; off += al(2 * act * es);
    const size_t o_kv1 = off; off += al(2 * act * es);
    const size_t o_acc = off; off += al(act * 4);
    const size_t o_lacc = off; off += al((size_t)BH * S * 4);
    const size_t o_part = off; off += al(act * es);
    const size_t o_lpart = off; off += al((size_t)BH * S * 4);
    const size_t o_stage = off; off += zig ? al(6 * (size_t)BH * C * D * es) : 0;
    const size_t o_rstage = off; off += zig ? al(6 * (size_t)BH * C * D * es) : 0;
    gae_status s;
    if ((s = ring_reserve(c, off)) != GAE_OK) return s;
    char *base = static_cast<char *>(c->buf);
    T *zq = reinterpret_cast<T *>(base + o_zq);
    T *kvb[2] = {reinterpret_cast<T *>(base + o_kv0), reinterpret_cast<T *>(base + o_kv1)};
    float *acc = reinterpret_cast<float *>(base + o_acc), *lacc = reinterpret_cast<float *>(base + o_lacc);
    T *part = reinterpret_cast<T *>(base + o_part);
    float *lpart = reinterpret_cast<float *>(base + o_lpart);
    char *stage = base + o_stage, *rstage = base + o_rstage;

    // Dense strides of the internal [BH, rows, D] buffers viewed as [B, H, rows, D].
    auto dense = [&](int64_t rows, int64_t out[3]) { out[0] = H * rows * D; out[1] = rows * D; out[2] = D; };
    int64_t zs[3];
    dense(S, zs);
    const T *srcs[3] = {static_cast<const T *>(a->q), static_cast<const T *>(a->k), static_cast<const T *>(a->v)};
    const int64_t *sstr[3] = {a->q_stride, a->k_stride, a->v_stride};
    T *dsts[3] = {zq, kvb[0], kvb[0] + act};

    // ---- layout in: zig-zag re-deal (or a plain copy into the buffers)
    if (!zig) {
        for (int i = 0; i < 3; ++i)
            if ((s = ring_copy(srcs[i], sstr[i], dsts[i], zs, B, H, S, D, st)) != GAE_OK) return s;
    } else {
        // my contiguous half i is global chunk 2r+i; its zig-zag owner and slot
        int64_t cs[3];
        dense(C, cs);
        for (int i = 0; i < 2; ++i) {
            const int ch = 2 * r + i, dst = ch < P ? ch : 2 * P - 1 - ch, slot = ch < P ? 0 : 1;
            if (dst != r) continue;
            for (int x = 0; x < 3; ++x)
                if ((s = ring_copy(srcs[x] + i * C * sstr[x][2], sstr[x], dsts[x] + slot * C * D, zs, B, H, C, D,
                                   st)) != GAE_OK)
                    return s;
        }
        // Remote moves: one send (my half i, packed q|k|v) and one receive
        // (my slot, packed) per moving chunk, all in one NCCL group.
        const size_t tri = (size_t)3 * BH * C * D;  // elements of one packed q|k|v chunk
        T *sendp[2] = {reinterpret_cast<T *>(stage), reinterpret_cast<T *>(stage) + tri};
        T *recvp = reinterpret_cast<T *>(rstage);
        for (int i = 0; i < 2; ++i) {
            const int ch = 2 * r + i, dst = ch < P ? ch : 2 * P - 1 - ch;
            if (dst == r) continue;
            for (int x = 0; x < 3; ++x)
                if ((s = ring_copy(srcs[x] + i * C * sstr[x][2], sstr[x], sendp[i] + (size_t)x * BH * C * D, cs, B,
                                   H, C, D, st)) != GAE_OK)
                    return s;
        }
        GAE_CUDA_TRY(cudaEventRecord(c->ev_a, st));
        GAE_CUDA_TRY(cudaStreamWaitEvent(c->comm_st, c->ev_a, 0));
        if ((s = nccl_settle(c, c->nc->GroupStart(), "re-deal group")) != GAE_OK) return s;
        for (int i = 0; i < 2; ++i) {
            const int ch = 2 * r + i, dst = ch < P ? ch : 2 * P - 1 - ch;
            if (dst != r &&
                (s = nccl_settle(c, c->nc->Send(sendp[i], tri * es, nt, dst, c->comm, c->comm_st), "re-deal send")) !=
                    GAE_OK)
                return s;
        }
        for (int slot = 0; slot < 2; ++slot) {
            const int ch = slot ? 2 * P - 1 - r : r, src = ch / 2;
            if (src != r && (s = nccl_settle(c, c->nc->Recv(recvp + slot * tri, tri * es, nt, src, c->comm, c->comm_st),
                                             "re-deal receive")) != GAE_OK)
                return s;
        }
        if ((s = nccl_settle(c, c->nc->GroupEnd(), "re-deal")) != GAE_OK) return s;
        GAE_CUDA_TRY(cudaEventRecord(c->ev_b, c->comm_st));
        GAE_CUDA_TRY(cudaStreamWaitEvent(st, c->ev_b, 0));
        for (int slot = 0; slot < 2; ++slot) {
            const int ch = slot ? 2 * P - 1 - r : r, src = ch / 2;
            if (src == r) continue;
            for (int x = 0; x < 3; ++x)
                if ((s = ring_copy(recvp + slot * tri + (size_t)x * BH * C * D, cs,
                                   dsts[x] + slot * C * D, zs, B, H, C, D, st)) != GAE_OK)
                    return s;
        }
    }

    prof.mark("re-deal in done", st);
    // ---- accumulator: O = 0, LSE = -inf
    GAE_CUDA_TRY(cudaMemsetAsync(acc, 0, act * 4, st));
    gae::ring_fill_kernel<<<256, 256, 0, st>>>(lacc, BH * S, -INFINITY);
    GAE_CUDA_TRY(cudaGetLastError());

    // ---- ring steps
    const size_t kv_bytes = 2 * act * es;
    for (int t = 0; t < P; ++t) {
        T *cur = kvb[t % 2], *nxt = kvb[(t + 1) % 2];
        if (t < P - 1) {
            // nxt was read by step t-1's launches (or the re-deal): wait for them
            GAE_CUDA_TRY(cudaEventRecord(c->ev_a, st));
            GAE_CUDA_TRY(cudaStreamWaitEvent(c->comm_st, c->ev_a, 0));
            if ((s = nccl_settle(c, c->nc->GroupStart(), "K/V exchange group")) != GAE_OK) return s;
            if ((s = nccl_settle(c, c->nc->Send(cur, kv_bytes, nt, (r + 1) % P, c->comm, c->comm_st),
                                 "K/V send")) != GAE_OK)
                return s;
            if ((s = nccl_settle(c, c->nc->Recv(nxt, kv_bytes, nt, (r - 1 + P) % P, c->comm, c->comm_st),
                                 "K/V receive")) != GAE_OK)
                return s;
            if ((s = nccl_settle(c, c->nc->GroupEnd(), "K/V exchange")) != GAE_OK) return s;
            GAE_CUDA_TRY(cudaEventRecord(c->ev_b, c->comm_st));
            prof.mark("  K/V exchange done", c->comm_st);
        }
        RingOp ops[2];
        const int n_ops = ring_plan(r, P, t, a->causal, zig, S, ops);
        for (int i = 0; i < n_ops; ++i) {
            const RingOp &op = ops[i];
            gae_attn_args la;
            memset(&la, 0, sizeof(la));
            int64_t ps[3];
            dense(op.q_rows, ps);
            la.q = zq + op.q_row0 * D;
            la.k = cur + op.kv_row0 * D;
            la.v = cur + act + op.kv_row0 * D;
            la.o = part;
            la.lse = lpart;
            la.batch = B; la.heads = H; la.seq_q = op.q_rows; la.seq_kv = op.kv_rows; la.head_dim = D;
            memcpy(la.q_stride, zs, sizeof zs); memcpy(la.k_stride, zs, sizeof zs);
            memcpy(la.v_stride, zs, sizeof zs); memcpy(la.o_stride, ps, sizeof ps);
            la.dtype = a->dtype;
            la.causal = op.causal;
            la.scale = a->scale;
            la.q_offset = op.q_pos;
            la.kv_offset = op.kv_pos;
            if ((s = launch_attn_tc(&la, st)) != GAE_OK) return s;
            const int64_t total = BH * op.q_rows;
            gae::ring_merge_kernel<T><<<(unsigned)((total + 7) / 8), 256, 0, st>>>(acc, lacc, part, lpart, op.q_rows,
                                                                                 S, op.q_row0, total, (int)D);
            GAE_CUDA_TRY(cudaGetLastError());
        }
        prof.mark("step compute done", st);
        if (t < P - 1) GAE_CUDA_TRY(cudaStreamWaitEvent(st, c->ev_b, 0));  // the next block has arrived
    }

    // ---- layout out
    T *out = static_cast<T *>(a->o);
    if (!zig) {
        if ((s = ring_copy(acc, zs, out, a->o_stride, B, H, S, D, st)) != GAE_OK) return s;
        if (a->lse) GAE_CUDA_TRY(cudaMemcpyAsync(a->lse, lacc, (size_t)BH * S * 4, cudaMemcpyDeviceToDevice, st));
    } else {
        int64_t cs[3];
        dense(C, cs);
        const int64_t ls3[3] = {H * S, S, 1}, lc3[3] = {H * C, C, 1};  // lse as [B, H, rows, 1]
        // my zig-zag slot -> contiguous owner ch/2, half ch%2
        T *sendp[2] = {reinterpret_cast<T *>(stage), reinterpret_cast<T *>(stage) + BH * C * D};
        float *lsend[2] = {reinterpret_cast<float *>(stage + 2 * (size_t)BH * C * D * es),
                           reinterpret_cast<float *>(stage + 2 * (size_t)BH * C * D * es) + BH * C};
        T *recvp[2] = {reinterpret_cast<T *>(rstage), reinterpret_cast<T *>(rstage) + BH * C * D};
        float *lrecv[2] = {reinterpret_cast<float *>(rstage + 2 * (size_t)BH * C * D * es),
                           reinterpret_cast<float *>(rstage + 2 * (size_t)BH * C * D * es) + BH * C};
        for (int slot = 0; slot < 2; ++slot) {
            const int ch = slot ? 2 * P - 1 - r : r, dst = ch / 2, half = ch % 2;
            if (dst == r) {
                if ((s = ring_copy(acc + slot * C * D, zs, out + half * C * a->o_stride[2], a->o_stride, B, H, C, D,
                                   st)) != GAE_OK)
                    return s;
                if (a->lse && (s = ring_copy(lacc + slot * C, ls3, a->lse + half * C, ls3, B, H, C, 1, st)) != GAE_OK)
                    return s;
            } else {
                if ((s = ring_copy(acc + slot * C * D, zs, sendp[slot], cs, B, H, C, D, st)) != GAE_OK) return s;
                if ((s = ring_copy(lacc + slot * C, ls3, lsend[slot], lc3, B, H, C, 1, st)) != GAE_OK) return s;
            }
        }
        GAE_CUDA_TRY(cudaEventRecord(c->ev_a, st));
        GAE_CUDA_TRY(cudaStreamWaitEvent(c->comm_st, c->ev_a, 0));
        if ((s = nccl_settle(c, c->nc->GroupStart(), "output re-deal group")) != GAE_OK) return s;
        for (int slot = 0; slot < 2; ++slot) {
            const int ch = slot ? 2 * P - 1 - r : r, dst = ch / 2;
            if (dst == r) continue;
            if ((s = nccl_settle(c, c->nc->Send(sendp[slot], (size_t)BH * C * D * es, nt, dst, c->comm, c->comm_st),
                                 "output send")) != GAE_OK ||
                (s = nccl_settle(c, c->nc->Send(lsend[slot], (size_t)BH * C * 4, nt, dst, c->comm, c->comm_st),
                                 "LSE send")) != GAE_OK)
                return s;
        }
        for (int half = 0; half < 2; ++half) {
            const int ch = 2 * r + half, src = ch < P ? ch : 2 * P - 1 - ch;
            if (src == r) continue;
            if ((s = nccl_settle(c, c->nc->Recv(recvp[half], (size_t)BH * C * D * es, nt, src, c->comm, c->comm_st),
                                 "output receive")) != GAE_OK ||
                (s = nccl_settle(c, c->nc->Recv(lrecv[half], (size_t)BH * C * 4, nt, src, c->comm, c->comm_st),
                                 "LSE receive")) != GAE_OK)
                return s;
        }
        if ((s = nccl_settle(c, c->nc->GroupEnd(), "output re-deal")) != GAE_OK) return s;
        GAE_CUDA_TRY(cudaEventRecord(c->ev_b, c->comm_st));
        GAE_CUDA_TRY(cudaStreamWaitEvent(st, c->ev_b, 0));
        for (int half = 0; half < 2; ++half) {
            const int ch = 2 * r + half, src = ch < P ? ch : 2 * P - 1 - ch;
            if (src == r) continue;
            if ((s = ring_copy(recvp[half], cs, out + half * C * a->o_stride[2], a->o_stride, B, H, C, D, st)) !=
                GAE_OK)
                return s;
            if (a->lse && (s = ring_copy(lrecv[half], lc3, a->lse + half * C, ls3, B, H, C, 1, st)) != GAE_OK)
                return s;
        }
    }
    prof.mark("re-deal out done", st);
    prof.report(c->rank);
    return GAE_OK;
}

gae_status ring_check_args(const gae_ring_ctx *c, const gae_attn_args *a, int balance, int *zig) {
    if (!c) return fail(GAE_ERR_INVALID_ARG, "ring context is NULL");
    if (!a) return fail(GAE_ERR_INVALID_ARG, "args is NULL");
    if (c->dead) return fail(GAE_ERR_COMM, "ring context was aborted after an earlier failure");
    if (a->dtype != GAE_DTYPE_BF16 && a->dtype != GAE_DTYPE_F16)
        return fail(GAE_ERR_UNSUPPORTED, "ring attention takes bf16 or f16 shards");
    if (a->seq_q != a->seq_kv) return fail(GAE_ERR_INVALID_ARG, "q and k/v shards must have the same length");
    if (a->q_offset != 0 || a->kv_offset != 0)
        return fail(GAE_ERR_INVALID_ARG, "ring attention derives positions from the rank; offsets must be 0");
    if (balance != GAE_RING_ZIGZAG && balance != GAE_RING_CONTIGUOUS)
        return fail(GAE_ERR_INVALID_ARG, "unknown balance %d", balance);
    *zig = (a->causal && balance == GAE_RING_ZIGZAG && c->world > 1) ? 1 : 0;
    if (*zig && (a->seq_q % 2)) return fail(GAE_ERR_INVALID_ARG, "zig-zag balance needs an even shard length");
    if (a->batch < 1 || a->heads < 1 || a->seq_q < 0 || (a->head_dim != 64 && a->head_dim != 128))
        return fail(GAE_ERR_UNSUPPORTED, "ring attention: head_dim 64 or 128 and positive batch/heads");
    if (a->batch * a->heads > 65535) return fail(GAE_ERR_UNSUPPORTED, "batch*heads above 65535");
    return GAE_OK;
}

}  // namespace
