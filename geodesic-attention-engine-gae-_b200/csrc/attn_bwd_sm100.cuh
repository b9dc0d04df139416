// attn_bwd_sm100.cuh -- exact attention backward (dQ, dK, dV) on the
// 5th-generation tensor cores.  The reference is inference-only; this is the
// training-side caller of the forward kernel (it consumes the forward's
// natural-log LSE and output).
//
// Math (P = softmax(scale * Q K^T) per row, recomputed from the LSE):
//   P    = exp(scale * S - lse)          S = Q K^T
//   dV   = P^T dO
//   dP   = dO V^T
//   dS   = P o (dP - Delta),             Delta = rowsum(dO o O)
//   dQ   = scale * dS K,   dK = scale * dS^T Q
//
// One CTA per (128-key tile j, batch*head): K_j and V_j stay in shared
// memory, dK_j and dV_j accumulate in TMEM across the CTA's query tiles
// (causal: tiles i >= j only).  Q_i streams through a two-stage ring, dO_i
// through one buffer that is reloaded as soon as dV_i has read it.  Per
// query tile the MMA warp issues
//   S = Q K^T, dP = dO V^T      (K-major x K-major)
//   dV += P^T dO                (P from shared memory read MN-major)
//   dK += dS^T Q                (dS likewise)
//   dQ  = dS K                  (dS K-major, K MN-major) into dP's columns
// in the order  dV_i, S_{i+1}, dK_i, dQ_i, then dP_{i+1} (two 64-column
// halves, each as soon as the drain has read that half of dQ_i) and dV_{i+1}
// in whichever order their inputs become ready.  S_{i+1} runs while the
// compute warps turn dP_i into dS_i, and they find it ready when they start
// P_{i+1}.  Two compute warpgroups turn S into P and dP into dS (bf16/f16
// into one shared tile in the 128-byte-swizzled layout both read directions
// share); a third warpgroup drains dQ_i from TMEM into a swizzled fp32
// staging tile (two halves) and adds it to an fp32 accumulator in global
// memory with TMA reduce-adds (cp.reduce.async.bulk.tensor, one per 128 x 32
// box): query tiles are shared by every key tile, so dQ is the one cross-CTA
// sum, and draining it stays off the compute warps' path.
//
// Reuse of the P/dS tile: dS_i overwrites P_i only after the dV_i MMA that
// reads P_i has completed; P_{i+1} overwrites dS_i only after dQ_i (issued
// after dK_i; tcgen05 MMAs of one thread complete in order) has completed.
//
// Warps: 0-7 compute (two warpgroups; thread = row of the 128-row tile and
// one half of its columns), 8-11 dQ drain, 12 TMA, 13 MMA (owns TMEM),
// 14 issues the dQ reduce-adds (so the drain warps never wait on them).
// TMEM columns: S [0,128), dP / dQ [128,256), dV [256,256+D), dK after it.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "sm100.cuh"

namespace gae {

struct AttnBwdParams {
    CUtensorMap tm_q, tm_k, tm_v, tm_do;  // dims {D, N, H, B}, box {64 elements, 128 rows}, 128B swizzle
    CUtensorMap tm_dq;                    // fp32 accumulator: dims {D, Nq, B*H}, box {32, 128, 1}, 128B swizzle
    const float *lse;                     // [B*H, Nq], natural log of sum exp(scale * s)
    const float *delta;                   // [B*H, Nq], rowsum(dO o O)
    float *dq_acc;                        // [B*H, Nq, D] fp32, zero on entry
    void *dk, *dv;
    int64_t dk_sb, dk_sh, dk_ss, dv_sb, dv_sh, dv_ss;  // element strides
    int B, H, Nq, Nkv, causal;
    float scale, scale_log2;
};

enum AttnBwdWaitSite : unsigned {
    kSiteBwdKV = 0x201,
    kSiteBwdQFull = 0x202,
    kSiteBwdQEmpty = 0x203,
    kSiteBwdS = 0x204,
    kSiteBwdDP = 0x205,
    kSiteBwdP = 0x206,
    kSiteBwdDS = 0x207,
    kSiteBwdDQ = 0x208,
    kSiteBwdDQFree = 0x209,
    kSiteBwdDone = 0x20a,
    kSiteBwdSmem = 0x20b,  // the aligned shared-memory payload did not fit (no wait involved)
};

// Cycle-stamp trace events of the backward kernel (diagnostics build only,
// same buffer as the forward's trace: event * kTraceTiles + query-tile step).
enum BwdTraceEvent : int {
    kBtS = 0, kBtPDone, kBtDP, kBtPC, kBtDSDone, kBtDQ, kBtDQDone,  // compute warp 0, lane 0
    kBtMmaP, kBtMmaDS, kBtMmaS, kBtMmaDP,                           // MMA issuer
    kBtTmaQ,                                                        // TMA producer: Q copy issued
};

template <int D>
struct AttnBwdCfg {
    static_assert(D == 64 || D == 128, "unsupported head_dim");
    static constexpr int kBox = 128 * 128;       // 128 rows x 128 bytes
    static constexpr int kPanels = D * 2 / 128;  // 64-element panels in a 128 x D tile
    static constexpr int kTile = kPanels * kBox;
    static constexpr int kPTile = 2 * kBox;      // 128 x 128, 16-bit
    static constexpr int kHalfD = D / 2;         // dQ is staged and drained in two halves
    static constexpr int kHalfBoxes = kHalfD / 32;  // fp32 boxes of 128 rows x 32 columns per half
    // K, V, Q[2], dO, P/dS, fp32 dQ staging (one half)
    static constexpr int kOffK = 0, kOffV = kTile, kOffQ = 2 * kTile, kOffDO = 4 * kTile;
    static constexpr int kOffPS = 5 * kTile, kOffDQ = kOffPS + kPTile, kOffBar = kOffDQ + kHalfBoxes * kBox;
    // kv, q_full[2], q_empty[2], do_full, do_empty, s, dp, p, p_consumed, ds, dq, dq_free[2], done,
    // staging_full, staging_free
    static constexpr int kNumBars = 18;
    static constexpr int kPayload = kOffBar + kNumBars * 8 + 16;
    // + slack for aligning the base to 1024 bytes (the swizzle atoms); the
    // kernel checks at run time that the aligned payload fits.
    static constexpr int kSmemBytes = (kPayload + 1024 < 227 * 1024) ? kPayload + 1024 : 227 * 1024;
    static constexpr uint32_t kColS = 0, kColDP = 128, kColDQ = 128, kColDV = 256, kColDK = 256 + D;
    static constexpr uint32_t kTmemCols = 512;
    static constexpr int kThreads = 480;
    static constexpr int kTmaWarp = 12, kMmaWarp = 13, kReduceWarp = 14;
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

// Tensor tile of global memory += shared tile (elementwise add, the map's
// element type), asynchronously on the TMA engine; elements outside the
// tensor are skipped.
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap *m, uint32_t src, int x, int y, int z) {
    asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(m)),
                 "r"(src), "r"(x), "r"(y), "r"(z)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// This thread's bulk operations have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// This thread's bulk operations have completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 16-bit pair <-> floats for the P tile kept in registers.
template <bool kBF16>
__device__ __forceinline__ void unpack2(uint32_t v, float &lo, float &hi) {
    if constexpr (kBF16) {
        lo = __uint_as_float(v << 16);
        hi = __uint_as_float(v & 0xffff0000u);
    } else {
        const __half2 h = *reinterpret_cast<const __half2 *>(&v);
        const float2 f = __half22float2(h);
        lo = f.x;
        hi = f.y;
    }
}

// Byte offset of the 16-byte chunk `ch` (0..15, 8 elements each) of row `row`
// in a 128 x 128 16-bit tile stored as two 64-column panels with the 128-byte
// swizzle (chunk index XOR row mod 8), the layout TMA writes for Q/K/V.
__device__ __forceinline__ uint32_t sw128_chunk(int row, int ch) {
    return (uint32_t)((ch >> 3) * (128 * 128) + row * 128 + (((ch & 7) ^ (row & 7)) << 4));
}

// Every kBwdPolyPeriod-th pair of probabilities is computed by the
// polynomial exp2 on the FMA pipe instead of the MUFU (0 = never): the P
// phase issues 16384 exponentials per tile against 16 MUFU results per
// cycle per SM.
#ifndef GAE_BWD_EMU_PERIOD
#define GAE_BWD_EMU_PERIOD 3
#endif
constexpr int kBwdPolyPeriod = GAE_BWD_EMU_PERIOD;

template <int D, bool kBF16>
__global__ void __launch_bounds__(480, 1) attn_bwd_sm100_kernel(const __grid_constant__ AttnBwdParams p) {
    using Cfg = AttnBwdCfg<D>;
    constexpr int kHalfD = Cfg::kHalfD;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t *smem = smem_raw + (base - raw_addr);
    if (base - raw_addr + Cfg::kPayload > (uint32_t)Cfg::kSmemBytes) {
        if (threadIdx.x == 0) record_error(kSiteBwdSmem);
        return;
    }
    const uint32_t sK = base + Cfg::kOffK, sV = base + Cfg::kOffV, sDO = base + Cfg::kOffDO;
    auto sQ = [&](int st) { return base + Cfg::kOffQ + st * Cfg::kTile; };
    const uint32_t sPS = base + Cfg::kOffPS, sDQ = base + Cfg::kOffDQ;
    const uint32_t sBar = base + Cfg::kOffBar;
    const uint32_t bar_kv = sBar;
    auto bar_q_full = [&](int st) { return sBar + 8u * (1 + st); };
    auto bar_q_empty = [&](int st) { return sBar + 8u * (3 + st); };
    const uint32_t bar_do_full = sBar + 40, bar_do_empty = sBar + 48;
    const uint32_t bar_s = sBar + 56, bar_dp = sBar + 64, bar_p = sBar + 72, bar_pc = sBar + 80;
    const uint32_t bar_ds = sBar + 88, bar_dq = sBar + 96, bar_done = sBar + 104;
    const uint32_t bar_st_full = sBar + 112, bar_st_free = sBar + 120;
    auto bar_dq_free = [&](int hh) { return sBar + 128u + 8u * hh; };  // half hh of dQ read from TMEM
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + Cfg::kOffBar + Cfg::kNumBars * 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int no_abort = 0;
#ifdef GAE_ATTN_TRACE
    unsigned long long *trace =
        (gae_attn_trace && blockIdx.x == gae_attn_trace_cta && blockIdx.y == 0) ? gae_attn_trace : nullptr;
#endif

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j = blockIdx.x, bh = blockIdx.y;
    const int b = bh / p.H, h = bh % p.H;
    const int n_q_tiles = (p.Nq + 127) / 128;
    const int i0 = p.causal ? j : 0;  // causal: Nq == Nkv and tile i sees key tile j only if i >= j
    const int n_it = n_q_tiles - i0;

    if (threadIdx.x == 0) {
        mbar_init(bar_kv, 1);
        for (int st = 0; st < 2; ++st) {
            mbar_init(bar_q_full(st), 1);
            mbar_init(bar_q_empty(st), 1);
        }
        mbar_init(bar_do_full, 1);
        mbar_init(bar_do_empty, 1);
        mbar_init(bar_s, 1);
        mbar_init(bar_dp, 1);
        mbar_init(bar_p, 256);
        mbar_init(bar_pc, 1);
        mbar_init(bar_ds, 256);
        mbar_init(bar_dq, 1);
        mbar_init(bar_dq_free(0), 128);
        mbar_init(bar_dq_free(1), 128);
        mbar_init(bar_done, 1);
        mbar_init(bar_st_full, 128);
        mbar_init(bar_st_free, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == Cfg::kMmaWarp) {
        tmem_alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == Cfg::kTmaWarp) {
        // ------------------------------------------------------ TMA producer
        if (lane == 0 && n_it > 0) {
            tma_prefetch_desc(&p.tm_q);
            tma_prefetch_desc(&p.tm_k);
            tma_prefetch_desc(&p.tm_v);
            tma_prefetch_desc(&p.tm_do);
            mbar_expect_tx(bar_kv, 2 * Cfg::kTile);
            for (int hf = 0; hf < Cfg::kPanels; ++hf) {
                tma_load_4d(sK + hf * Cfg::kBox, &p.tm_k, bar_kv, hf * 64, j * 128, h, b);
                tma_load_4d(sV + hf * Cfg::kBox, &p.tm_v, bar_kv, hf * 64, j * 128, h, b);
            }
            int n_q = 0, n_do = 0;  // copies issued
            for (int it = 0; it < n_it; ++it) {
                const int st = it & 1, row0 = (i0 + it) * 128;
                // Q_i reuses the stage of Q_{i-2}, free once dK_{i-2} completed.
                if (it >= 2 && !mbar_wait(bar_q_empty(st), ((it >> 1) - 1) & 1, kSiteBwdQEmpty, abort_flag)) break;
                GAE_TRACE(kBtTmaQ, it);
                mbar_expect_tx(bar_q_full(st), Cfg::kTile);
                for (int hf = 0; hf < Cfg::kPanels; ++hf)
                    tma_load_4d(sQ(st) + hf * Cfg::kBox, &p.tm_q, bar_q_full(st), hf * 64, row0, h, b);
                n_q = it + 1;
                // dO_i reuses dO_{i-1}'s buffer, free once dV_{i-1} completed.
                if (it > 0 && !mbar_wait(bar_do_empty, (it - 1) & 1, kSiteBwdQEmpty, abort_flag)) break;
                mbar_expect_tx(bar_do_full, Cfg::kTile);
                for (int hf = 0; hf < Cfg::kPanels; ++hf)
                    tma_load_4d(sDO + hf * Cfg::kBox, &p.tm_do, bar_do_full, hf * 64, row0, h, b);
                n_do = it + 1;
            }
            // Drain: the copies issued have landed before the CTA exits.
            mbar_wait(bar_kv, 0, kSiteBwdKV, &no_abort);
            for (int it = max(0, n_q - 2); it < n_q; ++it)
                mbar_wait(bar_q_full(it & 1), (it >> 1) & 1, kSiteBwdQFull, &no_abort);
            if (n_do > 0) mbar_wait(bar_do_full, (n_do - 1) & 1, kSiteBwdQFull, &no_abort);
        }
    } else if (warp == Cfg::kMmaWarp) {
        // ---------------------------------------------------------- MMA issuer
        if (lane == 0 && n_it > 0) {
            constexpr uint32_t id_qk = idesc_f16(128, 128, kBF16, false, false);
            constexpr uint32_t id_qk_half = idesc_f16(128, 64, kBF16, false, false);
            constexpr uint32_t id_t = idesc_f16(128, D, kBF16, true, true);    // P^T dO, dS^T Q
            constexpr uint32_t id_dq = idesc_f16(128, D, kBF16, false, true);  // dS K
            // 128 x 128 product over the head dimension, both operands K-major.
            auto mma_kk = [&](uint32_t d, uint32_t a, uint32_t bm) {
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * Cfg::kBox + (kk & 3) * 32;
                    umma_f16_ss(d, smem_desc_sw128(a + off, 16, 1024), smem_desc_sw128(bm + off, 16, 1024), id_qk,
                                kk > 0);
                }
            };
            bool ok = mbar_wait(bar_kv, 0, kSiteBwdKV, abort_flag) &&
                      mbar_wait(bar_q_full(0), 0, kSiteBwdQFull, abort_flag);
            if (ok) {
                tc_fence_after();
                mma_kk(tmem + Cfg::kColS, sQ(0), sK);
                umma_commit(bar_s);
                if ((ok = mbar_wait(bar_do_full, 0, kSiteBwdQFull, abort_flag))) {
                    tc_fence_after();
                    mma_kk(tmem + Cfg::kColDP, sDO, sV);
                    umma_commit(bar_dp);
                }
            }
            // dV_i: M = keys (MN-major in P), K = queries, N = D.
            auto issue_dv = [&](int it) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    umma_f16_ss(tmem + Cfg::kColDV, smem_desc_sw128(sPS + kk * 2048, Cfg::kBox, 1024),
                                smem_desc_sw128(sDO + kk * 2048, Cfg::kBox, 1024), id_t, (it > 0 || kk > 0));
                umma_commit(bar_pc);
            };
            // Half hh of dP = dO V^T: keys [64hh, 64hh + 64) into 64 columns.
            auto issue_dp_half = [&](int hh) {
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * Cfg::kBox + (kk & 3) * 32;
                    umma_f16_ss(tmem + Cfg::kColDP + 64 * hh, smem_desc_sw128(sDO + off, 16, 1024),
                                smem_desc_sw128(sV + hh * 64 * 128 + off, 16, 1024), id_qk_half, kk > 0);
                }
            };
            bool dv_issued = false;  // dV of the current tile already issued
            for (int it = 0; it < n_it && ok; ++it) {
                const int st = it & 1;
                const uint32_t ph = it & 1;
                if (!dv_issued) {
                    if (!(ok = mbar_wait(bar_p, ph, kSiteBwdP, abort_flag))) break;
                    GAE_TRACE(kBtMmaP, it);
                    tc_fence_after();
                    issue_dv(it);
                    umma_commit(bar_do_empty);  // dP_i and dV_i, dO_i's readers, are issued
                }
                dv_issued = false;
                // S_{i+1} while the compute warps form dS_i (S's columns were
                // released with P_i).
                if (it + 1 < n_it) {
                    const int sn = (it + 1) & 1;
                    if (!(ok = mbar_wait(bar_q_full(sn), ((it + 1) >> 1) & 1, kSiteBwdQFull, abort_flag))) break;
                    GAE_TRACE(kBtMmaS, it + 1);
                    tc_fence_after();
                    mma_kk(tmem + Cfg::kColS, sQ(sn), sK);
                    umma_commit(bar_s);
                }
                if (!(ok = mbar_wait(bar_ds, ph, kSiteBwdDS, abort_flag))) break;
                GAE_TRACE(kBtMmaDS, it);
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    umma_f16_ss(tmem + Cfg::kColDK, smem_desc_sw128(sPS + kk * 2048, Cfg::kBox, 1024),
                                smem_desc_sw128(sQ(st) + kk * 2048, Cfg::kBox, 1024), id_t, (it > 0 || kk > 0));
                umma_commit(bar_q_empty(st));
                // dQ = dS K: M = queries, K = keys (K-major in dS), N = D (MN-major in K).
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t off = (kk >> 2) * Cfg::kBox + (kk & 3) * 32;
                    umma_f16_ss(tmem + Cfg::kColDQ, smem_desc_sw128(sPS + off, 16, 1024),
                                smem_desc_sw128(sK + kk * 2048, Cfg::kBox, 1024), id_dq, kk > 0);
                }
                umma_commit(bar_dq);
                if (it + 1 < n_it) {
                    // dP_{i+1} (per half, once the drain has read that half of dQ_i
                    // and dO_{i+1} has landed) and dV_{i+1} (once P_{i+1} is in the
                    // tile), in whichever order they become ready.
                    const uint32_t pn = (it + 1) & 1;
                    bool dp_half[2] = {false, false};
                    const uint64_t t0 = globaltimer();
                    for (uint32_t spin = 0; !(dp_half[0] && dp_half[1]) || !dv_issued; ++spin) {
                        if (mbar_test(bar_do_full, pn)) {
                            bool progress = false;
                            for (int hh = 0; hh < 2; ++hh) {
                                if (dp_half[hh]) continue;
                                // dP half hh overwrites dQ columns [64hh, 64hh + 64) of D.
                                const bool free_ = (D == 128) ? mbar_test(bar_dq_free(hh), ph)
                                                   : (hh == 1 || (mbar_test(bar_dq_free(0), ph) &&
                                                                  mbar_test(bar_dq_free(1), ph)));
                                if (free_) {
                                    tc_fence_after();
                                    issue_dp_half(hh);
                                    dp_half[hh] = true;
                                    progress = true;
                                    if (dp_half[0] && dp_half[1]) {
                                        GAE_TRACE(kBtMmaDP, it + 1);
                                        umma_commit(bar_dp);
                                    }
                                }
                            }
                            if (!dv_issued && mbar_test(bar_p, pn)) {
                                GAE_TRACE(kBtMmaP, it + 1);
                                tc_fence_after();
                                issue_dv(it + 1);
                                dv_issued = true;
                                progress = true;
                            }
                            if (dp_half[0] && dp_half[1] && dv_issued) umma_commit(bar_do_empty);
                            if (progress) continue;
                        }
                        if ((spin & 63u) == 63u) {
                            if (*abort_flag) { ok = false; break; }
                            if (globaltimer() - t0 > GAE_WAIT_TIMEOUT_NS) {
                                *abort_flag = 1;
                                record_error(kSiteBwdDQFree);
                                ok = false;
                                break;
                            }
                        }
                    }
                }
            }
            umma_commit(bar_done);
            mbar_wait(bar_done, 0, kSiteBwdDone, &no_abort);
        }
    } else if (warp == Cfg::kReduceWarp) {
        // ------------------------------------------- dQ reduce-add issuer
        if (lane == 0) {
            bool ok = true;
            for (int n = 0; n < 2 * n_it && ok; ++n) {
                const int it = n >> 1, hh = n & 1;
                if (!(ok = mbar_wait(bar_st_full, n & 1, kSiteBwdDQ, abort_flag))) break;
                for (int c = 0; c < Cfg::kHalfBoxes; ++c)
                    tma_reduce_add_3d(&p.tm_dq, sDQ + c * Cfg::kBox, hh * kHalfD + c * 32, (i0 + it) * 128, bh);
                bulk_commit();
                bulk_wait_read();  // the staging tile may be rewritten
                mbar_arrive(bar_st_free);
            }
            bulk_wait_all();
        }
    } else if (warp >= 8 && warp < 12) {
        // ------------------------------------------------------- dQ drain
        const int row = (warp & 3) * 32 + lane;
        const uint32_t tDQ = tmem + ((uint32_t)((warp & 3) * 32) << 16) + Cfg::kColDQ;
        bool ok = n_it > 0;
        for (int it = 0; it < n_it && ok; ++it) {
            if (!(ok = mbar_wait(bar_dq, it & 1, kSiteBwdDQ, abort_flag))) break;
            if (row == 0) GAE_TRACE(kBtDQ, it);
            tc_fence_after();
            for (int hh = 0; hh < 2 && ok; ++hh) {
                const int n = 2 * it + hh;  // staging use
                uint32_t r[kHalfD];
#pragma unroll
                for (int c = 0; c < kHalfD / 32; ++c)
                    tmem_ld32(tDQ + hh * kHalfD + c * 32, *reinterpret_cast<uint32_t(*)[32]>(r + c * 32));
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(bar_dq_free(hh));  // this half of dP's columns may be rewritten
                if (row == 0 && hh == 1) GAE_TRACE(kBtDQDone, it);
                // The previous half's reduce-add has read the staging tile.
                if (n > 0 && !(ok = mbar_wait(bar_st_free, (n - 1) & 1, kSiteBwdDQFree, abort_flag))) break;
                // scale * dQ -> staging boxes (128 rows x 32 fp32, 128-byte swizzle:
                // conflict-free 16-byte stores).
#pragma unroll
                for (int c = 0; c < kHalfD / 32; ++c) {
                    const uint32_t box = sDQ + c * Cfg::kBox + row * 128;
#pragma unroll
                    for (int v = 0; v < 8; ++v)
                        st_shared_v4(box + ((v ^ (row & 7)) << 4),
                                     __float_as_uint(__uint_as_float(r[c * 32 + 4 * v]) * p.scale),
                                     __float_as_uint(__uint_as_float(r[c * 32 + 4 * v + 1]) * p.scale),
                                     __float_as_uint(__uint_as_float(r[c * 32 + 4 * v + 2]) * p.scale),
                                     __float_as_uint(__uint_as_float(r[c * 32 + 4 * v + 3]) * p.scale));
                }
                fence_proxy_async_smem();
                mbar_arrive(bar_st_full);
            }
        }
    } else {
        // ---------------------------------------------- compute warpgroups
        // Thread = (row, half): warps w and w+4 share TMEM lane quarter w % 4;
        // warpgroup g takes columns [64g, 64g + 64) of S/dP and half of dK/dV.
        const int g = warp >> 2;
        const int row = (warp & 3) * 32 + lane;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + lane_off + Cfg::kColS + 64 * g, tDP = tmem + lane_off + Cfg::kColDP + 64 * g;
        // Row statistics of the next query tile, loaded one step ahead.
        auto row_stats = [&](int it, float &lse2, float &dlt) {
            const int q = (i0 + it) * 128 + row;
            lse2 = INFINITY;  // +inf: the row contributes nothing
            dlt = 0.f;
            if (it < n_it && q < p.Nq) {
                const float l = __ldg(p.lse + (int64_t)bh * p.Nq + q);
                if (l != -INFINITY) lse2 = l * 1.4426950408889634f;
                dlt = __ldg(p.delta + (int64_t)bh * p.Nq + q);
            }
        };
        float lse2_n, dlt_n;
        row_stats(0, lse2_n, dlt_n);
        bool ok = n_it > 0;
        for (int it = 0; it < n_it && ok; ++it) {
            const uint32_t ph = it & 1;
            const int q = (i0 + it) * 128 + row;
            const float lse2 = lse2_n, dlt = dlt_n;
            row_stats(it + 1, lse2_n, dlt_n);
            // Keys of this tile (and this half) the row may see: [0, lim).
            int lim = min(128, p.Nkv - j * 128);
            if (p.causal) lim = min(lim, max(0, q - j * 128 + 1));
            lim -= 64 * g;

            if (!(ok = mbar_wait(bar_s, ph, kSiteBwdS, abort_flag))) break;
            if (row == 0 && g == 0) GAE_TRACE(kBtS, it);
            tc_fence_after();
            uint32_t pk[32];
            {
                uint32_t r0[32], r1[32];
                tmem_ld32(tS, r0);
                tmem_ld32(tS + 32, r1);
                tmem_wait_ld();
                const uint64_t sl2x2 = f2_pack(p.scale_log2, p.scale_log2), nl2 = f2_pack(-lse2, -lse2);
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const uint32_t *r = (e < 16) ? r0 : r1;
                    const int ee = e & 15, k0 = 2 * e;
                    const uint64_t x = f2_fma(f2_pack(__uint_as_float(r[2 * ee]), __uint_as_float(r[2 * ee + 1])),
                                              sl2x2, nl2);
                    float p0, p1;
                    if (kBwdPolyPeriod > 0 && e % kBwdPolyPeriod == kBwdPolyPeriod - 1) {
                        exp2_poly_x2(x, p0, p1);  // this pair on the FMA pipe
                    } else {
                        float x0, x1;
                        f2_unpack(x, x0, x1);
                        p0 = ex2_approx(x0);
                        p1 = ex2_approx(x1);
                    }
                    p0 = (k0 < lim) ? p0 : 0.f;
                    p1 = (k0 + 1 < lim) ? p1 : 0.f;
                    pk[e] = kBF16 ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
                }
            }
            // dS_{i-1} stays in the tile until dQ_{i-1}, its last reader, completed.
            if (it > 0 && !(ok = mbar_wait(bar_dq, (it - 1) & 1, kSiteBwdDQ, abort_flag))) break;
#pragma unroll
            for (int c = 0; c < 8; ++c)
                st_shared_v4(sPS + sw128_chunk(row, 8 * g + c), pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(bar_p);
            if (row == 0 && g == 0) GAE_TRACE(kBtPDone, it);

            if (!(ok = mbar_wait(bar_dp, ph, kSiteBwdDP, abort_flag))) break;
            if (row == 0 && g == 0) GAE_TRACE(kBtDP, it);
            tc_fence_after();
            {
                uint32_t r0[32], r1[32];
                tmem_ld32(tDP, r0);
                tmem_ld32(tDP + 32, r1);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    float p0, p1;
                    unpack2<kBF16>(pk[e], p0, p1);
                    pk[e] = kBF16 ? pack_bf16x2(p0 * (__uint_as_float(r0[2 * e]) - dlt),
                                                p1 * (__uint_as_float(r0[2 * e + 1]) - dlt))
                                  : pack_f16x2(p0 * (__uint_as_float(r0[2 * e]) - dlt),
                                               p1 * (__uint_as_float(r0[2 * e + 1]) - dlt));
                    unpack2<kBF16>(pk[16 + e], p0, p1);
                    pk[16 + e] = kBF16 ? pack_bf16x2(p0 * (__uint_as_float(r1[2 * e]) - dlt),
                                                     p1 * (__uint_as_float(r1[2 * e + 1]) - dlt))
                                       : pack_f16x2(p0 * (__uint_as_float(r1[2 * e]) - dlt),
                                                    p1 * (__uint_as_float(r1[2 * e + 1]) - dlt));
                }
            }
            tc_fence_before();
            // P_i stays in the tile until the dV_i MMA that reads it has completed.
            if (!(ok = mbar_wait(bar_pc, ph, kSiteBwdP, abort_flag))) break;
            if (row == 0 && g == 0) GAE_TRACE(kBtPC, it);
#pragma unroll
            for (int c = 0; c < 8; ++c)
                st_shared_v4(sPS + sw128_chunk(row, 8 * g + c), pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
            fence_proxy_async_smem();
            mbar_arrive(bar_ds);
            if (row == 0 && g == 0) GAE_TRACE(kBtDSDone, it);
        }
        // Epilogue: this half of dV and scale * dK of the key tile -> global.
        if (ok && mbar_wait(bar_done, 0, kSiteBwdDone, abort_flag)) {
            tc_fence_after();
            const int key = j * 128 + row;
            const bool kvalid = key < p.Nkv;
            for (int t = 0; t < 2; ++t) {
                const uint32_t tc = tmem + lane_off + (t ? Cfg::kColDK : Cfg::kColDV) + kHalfD * g;
                const float mul = t ? p.scale : 1.f;
                char *dst = reinterpret_cast<char *>(t ? p.dk : p.dv) +
                            2 * (t ? (b * p.dk_sb + h * p.dk_sh + (int64_t)key * p.dk_ss)
                                   : (b * p.dv_sb + h * p.dv_sh + (int64_t)key * p.dv_ss)) +
                            2 * kHalfD * g;
#pragma unroll
                for (int c = 0; c < kHalfD / 32; ++c) {
                    uint32_t r[32], pkd[16];
                    tmem_ld32(tc + c * 32, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const float a0 = __uint_as_float(r[2 * e]) * mul, a1 = __uint_as_float(r[2 * e + 1]) * mul;
                        pkd[e] = kBF16 ? pack_bf16x2(a0, a1) : pack_f16x2(a0, a1);
                    }
                    if (kvalid) {
                        uint4 *d4 = reinterpret_cast<uint4 *>(dst + c * 64);
#pragma unroll
                        for (int v = 0; v < 4; ++v)
                            d4[v] = make_uint4(pkd[4 * v], pkd[4 * v + 1], pkd[4 * v + 2], pkd[4 * v + 3]);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == Cfg::kMmaWarp) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
    }
}

// Delta[bh][q] = sum_d dO[q][d] * O[q][d] (fp32), one warp per row.
template <typename T>
__global__ void attn_bwd_delta_kernel(const T *o, const T *dout, float *delta, int B, int H, int N, int D,
                                      int64_t o_sb, int64_t o_sh, int64_t o_ss, int64_t d_sb, int64_t d_sh,
                                      int64_t d_ss) {
    const int64_t rowid = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (rowid >= (int64_t)B * H * N) return;
    const int q = (int)(rowid % N);
    const int bh = (int)(rowid / N), b = bh / H, h = bh % H;
    const T *orow = o + b * o_sb + h * o_sh + (int64_t)q * o_ss;
    const T *drow = dout + b * d_sb + h * d_sh + (int64_t)q * d_ss;
    float s = 0.f;
    for (int c = lane * 8; c < D; c += 256) {
        const uint4 ov = *reinterpret_cast<const uint4 *>(orow + c);
        const uint4 dv = *reinterpret_cast<const uint4 *>(drow + c);
        const uint32_t oa[4] = {ov.x, ov.y, ov.z, ov.w}, da[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            float o0, o1, d0, d1;
            unpack2<std::is_same<T, __nv_bfloat16>::value>(oa[u], o0, o1);
            unpack2<std::is_same<T, __nv_bfloat16>::value>(da[u], d0, d1);
            s = fmaf(o0, d0, s);
            s = fmaf(o1, d1, s);
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) delta[rowid] = s;
}

// dQ (16-bit, strided) from the fp32 accumulator [B*H, N, D].
template <typename T>
__global__ void attn_bwd_dq_kernel(const float *acc, T *dq, int B, int H, int N, int D, int64_t sb, int64_t sh,
                                   int64_t ss) {
    const int64_t i4 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t total4 = (int64_t)B * H * N * D / 4;
    if (i4 >= total4) return;
    const int64_t i = 4 * i4;
    const int d = (int)(i % D);
    const int64_t rowid = i / D;
    const int q = (int)(rowid % N);
    const int bh = (int)(rowid / N), b = bh / H, h = bh % H;
    const float4 v = *reinterpret_cast<const float4 *>(acc + i);
    T *dst = dq + b * sb + h * sh + (int64_t)q * ss + d;
    uint32_t lo, hi;
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        lo = pack_bf16x2(v.x, v.y);
        hi = pack_bf16x2(v.z, v.w);
    } else {
        lo = pack_f16x2(v.x, v.y);
        hi = pack_f16x2(v.z, v.w);
    }
    *reinterpret_cast<uint2 *>(dst) = make_uint2(lo, hi);
}

}  // namespace gae
