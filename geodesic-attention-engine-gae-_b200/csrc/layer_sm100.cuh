// layer_sm100.cuh -- kernels of the fused pre-norm transformer layer on B200.
//
// The reference's fused layer is cuda_src/waller_fused_layer.cu:64-247 (one
// thread per token through int8 attention, RMSNorm and a small MLP) and its
// crate API is ate::TransformerBlock (rust_src/src/transformer.rs:87-120) built
// from layernorm (layernorm.rs:20-47), mlp_block (mlp.rs:7-36) and the tanh
// GELU (activations.rs:5-7).  Here the layer is a real GPT-2 pre-norm block at
// tensor-core scale:
//   * linear_kernel: persistent warp-specialised GEMM Y = X W^T on tcgen05.
//     X [M, K] and W [N, K] bf16, both K-major, arrive by TMA (128-byte
//     swizzle) into a 4-stage shared-memory ring; one thread issues
//     128x256x16 MMAs into one of two TMEM accumulators (2 x 256 columns);
//     eight epilogue warps drain the other accumulator (thread = output row,
//     two warps per row quarter, one per column half)
//     and fuse bias, tanh-GELU or the residual add, writing bf16.
//   * layernorm_kernel: one warp per row (persistent warps, gamma/beta
//     in registers), 16-byte vector loads, fp32
//     statistics (population variance, eps inside the square root, as
//     layernorm.rs:6-17), optional fused residual add.
#pragma once
#include "sm100.cuh"

namespace gae {

enum LinearEpilogue : int { kEpiBias = 0, kEpiBiasGelu = 1, kEpiBiasResidual = 2 };

struct LinearParams {
    CUtensorMap tm_a;  // X: dims {K, M}, box {64, 128}
    CUtensorMap tm_b;  // W: dims {K, N}, box {64, 256}
    __nv_bfloat16 *y;  // [M, N], row stride ldy
    const float *bias;                 // [N] or null
    const __nv_bfloat16 *res;          // [M, N] (row stride ldr) for kEpiBiasResidual
    int M, N, K;
    int64_t ldy, ldr;
    int epi;
    int tiles_m, tiles_n;
};

struct LinearCfg {
    static constexpr int BM = 128, BN = 256, BK = 64;
    static constexpr int kStages = 4;
    static constexpr int kABytes = BM * BK * 2;   // 16 KB
    static constexpr int kBBytes = BN * BK * 2;   // 32 KB
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kBarOffset = kStages * kStageBytes;
    // full[S], empty[S], acc_full[2], acc_empty[2], done
    static constexpr int kNumBars = 2 * kStages + 5;
    static constexpr int kSmemBytes = kBarOffset + kNumBars * 8 + 16 + 1024;
    static constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
};

enum LinearWaitSite : unsigned {
    kSiteLinFull = 0x301, kSiteLinEmpty = 0x302, kSiteLinAccFull = 0x303, kSiteLinAccEmpty = 0x304,
    kSiteLinDone = 0x305,
};

// 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), the reference's GELU
// (rust_src/src/activations.rs:5-7), with the hardware tanh approximation.
__device__ __forceinline__ float gelu_tanh(float x) {
    const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
    const float u = k0 * fmaf(0.044715f * x, x * x, x);
    float t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
    return 0.5f * x * (1.f + t);
}

__global__ void __launch_bounds__(320, 1) linear_kernel(const __grid_constant__ LinearParams p) {
    using Cfg = LinearCfg;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t *smem = smem_raw + (base - raw_addr);
    const uint32_t sBar = base + Cfg::kBarOffset;
    auto bar_full = [&](int s) { return sBar + 8u * s; };
    auto bar_empty = [&](int s) { return sBar + 8u * (Cfg::kStages + s); };
    auto bar_acc_full = [&](int b) { return sBar + 8u * (2 * Cfg::kStages + b); };
    auto bar_acc_empty = [&](int b) { return sBar + 8u * (2 * Cfg::kStages + 2 + b); };
    const uint32_t bar_done = sBar + 8u * (2 * Cfg::kStages + 4);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + Cfg::kBarOffset + Cfg::kNumBars * 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int no_abort = 0;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tiles = p.tiles_m * p.tiles_n;
    const int kb_count = p.K / Cfg::BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::kStages; ++s) {
            mbar_init(bar_full(s), 1);
            mbar_init(bar_empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar_acc_full(b), 1);
            mbar_init(bar_acc_empty(b), 256);
        }
        mbar_init(bar_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Tiles of this CTA: blockIdx.x, blockIdx.x + gridDim.x, ...  N-fastest
    // raster, so CTAs running at the same time share rows of X in L2.
    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&p.tm_a);
            tma_prefetch_desc(&p.tm_b);
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
                const int m0 = (t / p.tiles_n) * Cfg::BM, n0 = (t % p.tiles_n) * Cfg::BN;
                for (int kb = 0; kb < kb_count; ++kb, ++it) {
                    const int s = it % Cfg::kStages, use = it / Cfg::kStages;
                    if (use > 0 && !(ok = mbar_wait(bar_empty(s), (use - 1) & 1, kSiteLinEmpty, abort_flag)))
                        break;
                    const uint32_t dst = base + s * Cfg::kStageBytes;
                    mbar_expect_tx(bar_full(s), Cfg::kStageBytes);
                    tma_load_2d(dst, &p.tm_a, bar_full(s), kb * Cfg::BK, m0);
                    tma_load_2d(dst + Cfg::kABytes, &p.tm_b, bar_full(s), kb * Cfg::BK, n0);
                }
            }
            // Drain the copies still in flight (bounded).
            for (int i = max(0, it - Cfg::kStages); i < it; ++i)
                mbar_wait(bar_full(i % Cfg::kStages), (i / Cfg::kStages) & 1, kSiteLinFull, &no_abort);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(Cfg::BM, Cfg::BN, true, false, false);
            int it = 0, local = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++local) {
                const int b = local & 1, use = local >> 1;
                if (use > 0 && !(ok = mbar_wait(bar_acc_empty(b), (use - 1) & 1, kSiteLinAccEmpty, abort_flag)))
                    break;
                tc_fence_after();
                const uint32_t acc = tmem + b * Cfg::BN;
                for (int kb = 0; kb < kb_count; ++kb, ++it) {
                    const int s = it % Cfg::kStages;
                    if (!(ok = mbar_wait(bar_full(s), (it / Cfg::kStages) & 1, kSiteLinFull, abort_flag))) break;
                    tc_fence_after();
                    const uint32_t sa = base + s * Cfg::kStageBytes, sb = sa + Cfg::kABytes;
#pragma unroll
                    for (int kk = 0; kk < Cfg::BK / 16; ++kk)
                        umma_f16_ss(acc, smem_desc_sw128(sa + kk * 32, 16, 1024),
                                    smem_desc_sw128(sb + kk * 32, 16, 1024), idesc,
                                    (kb > 0 || kk > 0) ? 1u : 0u);
                    umma_commit(bar_empty(s));
                }
                if (ok) umma_commit(bar_acc_full(b));
            }
            // Drain: all issued MMAs complete before TMEM is released (bounded,
            // not cut short by the abort flag).
            umma_commit(bar_done);
            mbar_wait(bar_done, 0, kSiteLinDone, &no_abort);
        }
    } else {
        // Epilogue warps 2-9: TMEM lane quarter = warp % 4 (thread = row); warps
        // 2-5 take columns [0, 128) of the tile, warps 6-9 columns [128, 256).
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        int local = 0;
        for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++local) {
            const int b = local & 1, use = local >> 1;
            if (!mbar_wait(bar_acc_full(b), use & 1, kSiteLinAccFull, abort_flag)) break;
            tc_fence_after();
            const int m = (t / p.tiles_n) * Cfg::BM + row;
            const int n0 = (t % p.tiles_n) * Cfg::BN;
            const bool valid = m < p.M;
            __nv_bfloat16 *yrow = p.y + (int64_t)m * p.ldy + n0;
            const __nv_bfloat16 *rrow = (p.epi == kEpiBiasResidual) ? p.res + (int64_t)m * p.ldr + n0 : nullptr;
#pragma unroll 1
            for (int cc = 0; cc < 2; ++cc) {
                // 64 columns per TMEM wait.
                uint32_t r[2][32];
                const int c0 = half * 4 + cc * 2;
                tmem_ld32(tmem + lane_off + b * Cfg::BN + c0 * 32, r[0]);
                tmem_ld32(tmem + lane_off + b * Cfg::BN + c0 * 32 + 32, r[1]);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                const int c = c0 + i;
                float v[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[i][e]);
                if (p.bias) {
                    const float4 *bp = reinterpret_cast<const float4 *>(p.bias + n0 + c * 32);
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float4 bb = __ldg(bp + q);
                        v[4 * q] += bb.x; v[4 * q + 1] += bb.y; v[4 * q + 2] += bb.z; v[4 * q + 3] += bb.w;
                    }
                }
                if (p.epi == kEpiBiasGelu) {
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] = gelu_tanh(v[e]);
                } else if (p.epi == kEpiBiasResidual && valid) {
                    const uint4 *rp = reinterpret_cast<const uint4 *>(rrow + c * 32);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint4 rv = rp[q];
                        const uint32_t w4[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            v[8 * q + 2 * u] += __uint_as_float(w4[u] << 16);
                            v[8 * q + 2 * u + 1] += __uint_as_float(w4[u] & 0xffff0000u);
                        }
                    }
                }
                if (valid) {
                    uint4 *dst = reinterpret_cast<uint4 *>(yrow + c * 32);
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        dst[q] = make_uint4(pack_bf16x2(v[8 * q], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                                            pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
                }
                }
            }
            tc_fence_before();
            mbar_arrive(bar_acc_empty(b));
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}


// ------------------------------------------------------- 2-SM linear layer
// The same GEMM with the epilogues above on CTA pairs (a cluster of 2): the
// pair computes a 256 x 256 tile with tcgen05.mma.cta_group::2 (M = 256).
// Each CTA holds its own 128 rows of X and its own 128 rows (one N half) of
// W per stage, so each SM streams half as many weight bytes per FLOP as the
// one-SM kernel and a stage is 32 KB, leaving room for 6 stages.  The
// leader CTA (rank 0) owns the pipeline: both CTAs' TMA copies complete on
// its "full" barriers, its one thread issues the MMAs, and its commits reach
// the "empty" and "accumulator full" barriers of both CTAs.  Each CTA's
// TMEM holds its 128 rows of the two 256-column accumulators; each CTA's
// eight epilogue warps drain its rows and arrive on the leader's
// "accumulator empty" barrier.
#ifndef GAE_LINEAR_RELAXED_ARRIVE
#define GAE_LINEAR_RELAXED_ARRIVE 1
#endif
struct Linear2Cfg {
    static constexpr int BM = 256, BN = 256, BK = 64;  // pair tile
    static constexpr int kStages = 6;
    static constexpr int kABytes = 128 * BK * 2;        // this CTA's 128 rows of X
    static constexpr int kBBytes = 128 * BK * 2;        // this CTA's N half of W
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kBarOffset = kStages * kStageBytes;
    // full[S], empty[S], acc_full[2], acc_empty[2], done
    static constexpr int kNumBars = 2 * kStages + 5;
    static constexpr int kSmemBytes = kBarOffset + kNumBars * 8 + 16 + 1024;
    static constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(320, 1)
    linear2_kernel(const __grid_constant__ LinearParams p) {
    using Cfg = Linear2Cfg;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t *smem = smem_raw + (base - raw_addr);
    const uint32_t sBar = base + Cfg::kBarOffset;
    auto bar_full = [&](int s) { return sBar + 8u * s; };
    auto bar_empty = [&](int s) { return sBar + 8u * (Cfg::kStages + s); };
    auto bar_acc_full = [&](int b) { return sBar + 8u * (2 * Cfg::kStages + b); };
    auto bar_acc_empty = [&](int b) { return sBar + 8u * (2 * Cfg::kStages + 2 + b); };
    const uint32_t bar_done = sBar + 8u * (2 * Cfg::kStages + 4);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + Cfg::kBarOffset + Cfg::kNumBars * 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int no_abort = 0;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
    const int tiles_m = (p.M + Cfg::BM - 1) / Cfg::BM, tiles_n = p.N / Cfg::BN;
    const int n_tiles = tiles_m * tiles_n;
    const int kb_count = p.K / Cfg::BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < Cfg::kStages; ++s) {
            mbar_init(bar_full(s), 1);
            mbar_init(bar_empty(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(bar_acc_full(b), 1);
            mbar_init(bar_acc_empty(b), 2 * 256);  // epilogue threads of both CTAs
        }
        mbar_init(bar_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_slot), 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised before any remote use
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&p.tm_a);
            tma_prefetch_desc(&p.tm_b);
            int it = 0;
            bool ok = true;
            for (int t = pair; t < n_tiles && ok; t += n_pairs) {
                const int m0 = (t / tiles_n) * Cfg::BM + (int)rank * 128;
                const int n0 = (t % tiles_n) * Cfg::BN + (int)rank * 128;
                for (int kb = 0; kb < kb_count; ++kb, ++it) {
                    const int s = it % Cfg::kStages, use = it / Cfg::kStages;
                    if (use > 0 && !(ok = mbar_wait(bar_empty(s), (use - 1) & 1, kSiteLinEmpty, abort_flag)))
                        break;
                    if (leader) mbar_expect_tx(bar_full(s), 2 * Cfg::kStageBytes);
                    const uint32_t full0 = mapa_shared(bar_full(s), 0);
                    const uint32_t dst = base + s * Cfg::kStageBytes;
                    tma_load_2d_pair(dst, &p.tm_a, full0, kb * Cfg::BK, m0);
                    tma_load_2d_pair(dst + Cfg::kABytes, &p.tm_b, full0, kb * Cfg::BK, n0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = idesc_f16(Cfg::BM, Cfg::BN, true, false, false);
            int it = 0, local = 0;
            bool ok = true;
            for (int t = pair; t < n_tiles && ok; t += n_pairs, ++local) {
                const int b = local & 1, use = local >> 1;
                if (use > 0 && !(ok = mbar_wait(bar_acc_empty(b), (use - 1) & 1, kSiteLinAccEmpty, abort_flag)))
                    break;
                tc_fence_after();
                const uint32_t acc = tmem + b * Cfg::BN;
                for (int kb = 0; kb < kb_count; ++kb, ++it) {
                    const int s = it % Cfg::kStages;
                    if (!(ok = mbar_wait(bar_full(s), (it / Cfg::kStages) & 1, kSiteLinFull, abort_flag))) break;
                    tc_fence_after();
                    const uint32_t sa = base + s * Cfg::kStageBytes, sb = sa + Cfg::kABytes;
#pragma unroll
                    for (int kk = 0; kk < Cfg::BK / 16; ++kk)
                        umma_f16_ss_pair(acc, smem_desc_sw128(sa + kk * 32, 16, 1024),
                                         smem_desc_sw128(sb + kk * 32, 16, 1024), idesc,
                                         (kb > 0 || kk > 0) ? 1u : 0u);
                    umma_commit_pair_both(bar_empty(s));
                }
                if (ok) umma_commit_pair_both(bar_acc_full(b));
            }
            // Drain: all issued MMAs complete before TMEM is released.
            umma_commit_pair(bar_done);
            mbar_wait(bar_done, 0, kSiteLinDone, &no_abort);
        }
    } else {
        // Epilogue warps 2-9, as in linear_kernel, on this CTA's 128 rows.
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        int local = 0;
        for (int t = pair; t < n_tiles; t += n_pairs, ++local) {
            const int b = local & 1, use = local >> 1;
            if (!mbar_wait(bar_acc_full(b), use & 1, kSiteLinAccFull, abort_flag)) break;
            tc_fence_after();
            const int m = (t / tiles_n) * Cfg::BM + (int)rank * 128 + row;
            const int n0 = (t % tiles_n) * Cfg::BN;
            const bool valid = m < p.M;
            __nv_bfloat16 *yrow = p.y + (int64_t)m * p.ldy + n0;
            const __nv_bfloat16 *rrow = (p.epi == kEpiBiasResidual) ? p.res + (int64_t)m * p.ldr + n0 : nullptr;
#pragma unroll 1
            for (int cc = 0; cc < 2; ++cc) {
                uint32_t r[2][32];
                const int c0 = half * 4 + cc * 2;
                tmem_ld32(tmem + lane_off + b * Cfg::BN + c0 * 32, r[0]);
                tmem_ld32(tmem + lane_off + b * Cfg::BN + c0 * 32 + 32, r[1]);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const int c = c0 + i;
                    float v[32];
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[i][e]);
                    if (p.bias) {
                        const float4 *bp = reinterpret_cast<const float4 *>(p.bias + n0 + c * 32);
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            const float4 bb = __ldg(bp + q);
                            v[4 * q] += bb.x; v[4 * q + 1] += bb.y; v[4 * q + 2] += bb.z; v[4 * q + 3] += bb.w;
                        }
                    }
                    if (p.epi == kEpiBiasGelu) {
#pragma unroll
                        for (int e = 0; e < 32; ++e) v[e] = gelu_tanh(v[e]);
                    } else if (p.epi == kEpiBiasResidual && valid) {
                        const uint4 *rp = reinterpret_cast<const uint4 *>(rrow + c * 32);
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const uint4 rv = rp[q];
                            const uint32_t w4[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                v[8 * q + 2 * u] += __uint_as_float(w4[u] << 16);
                                v[8 * q + 2 * u + 1] += __uint_as_float(w4[u] & 0xffff0000u);
                            }
                        }
                    }
                    if (valid) {
                        uint4 *dst = reinterpret_cast<uint4 *>(yrow + c * 32);
#pragma unroll
                        for (int q = 0; q < 4; ++q)
                            dst[q] = make_uint4(pack_bf16x2(v[8 * q], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                                                pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
                    }
                }
            }
            // The accumulator is free once this thread's TMEM reads are done
            // (each tcgen05.ld was waited for); its global stores need not be
            // ordered before the MMA warp reuses the accumulator, so a relaxed
            // arrive (a release would wait for the stores to complete).
            tc_fence_before();
#if GAE_LINEAR_RELAXED_ARRIVE
            mbar_arrive_remote_relaxed(mapa_shared(bar_acc_empty(b), 0));
#else
            mbar_arrive_remote(mapa_shared(bar_acc_empty(b), 0));
#endif
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the leader's MMAs no longer read either CTA's smem or TMEM
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
}

// ------------------------------------------------------------- LayerNorm
// One warp per row.  s = x (+ res, rounded to bf16 and written to sum_out);
// y = (s - mean) / sqrt(var + eps) * gamma + beta with the population
// variance; statistics in fp32 by two passes over registers.  kPerLane
// 16-byte chunks per lane (d <= 256 * kPerLane) are held in registers, so the
// instantiation is picked by row width to keep registers low and many rows in
// flight per SM (the kernel is HBM-bound).
constexpr int kLnMaxChunks = 16;  // 16 x 8 x 32 = 4096 elements per row at most

// Persistent rows: each warp walks rows warp_id, warp_id + total_warps, ...
// with gamma and beta held in registers for all of them (loaded once), and
// the next row's 16-byte chunks loaded before the current row is reduced.
template <int kPerLane>
__global__ void __launch_bounds__(256) layernorm_kernel(const __nv_bfloat16 *x, const __nv_bfloat16 *res,
                                                        __nv_bfloat16 *sum_out, __nv_bfloat16 *y,
                                                        const float *gamma, const float *beta,
                                                        int64_t rows, int D, float eps) {
    const int lane = threadIdx.x & 31;
    const int64_t warps_total = (int64_t)gridDim.x * (blockDim.x >> 5);
    int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int chunks = D / 8;  // 16-byte chunks per row
    if (row >= rows) return;
    float g[kPerLane][8], bb[kPerLane][8];  // this lane's gamma/beta, for all of the warp's rows
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
        const int c = lane + 32 * i;
        if (c < chunks) {
            const float4 g0 = __ldg(reinterpret_cast<const float4 *>(gamma) + 2 * c);
            const float4 g1 = __ldg(reinterpret_cast<const float4 *>(gamma) + 2 * c + 1);
            const float4 b0 = __ldg(reinterpret_cast<const float4 *>(beta) + 2 * c);
            const float4 b1 = __ldg(reinterpret_cast<const float4 *>(beta) + 2 * c + 1);
            g[i][0] = g0.x; g[i][1] = g0.y; g[i][2] = g0.z; g[i][3] = g0.w;
            g[i][4] = g1.x; g[i][5] = g1.y; g[i][6] = g1.z; g[i][7] = g1.w;
            bb[i][0] = b0.x; bb[i][1] = b0.y; bb[i][2] = b0.z; bb[i][3] = b0.w;
            bb[i][4] = b1.x; bb[i][5] = b1.y; bb[i][6] = b1.z; bb[i][7] = b1.w;
        }
    }
    uint4 raw[kPerLane], rraw[kPerLane];
    auto load_row = [&](int64_t r) {
        const uint4 *xr = reinterpret_cast<const uint4 *>(x + r * D);
        const uint4 *rr = res ? reinterpret_cast<const uint4 *>(res + r * D) : nullptr;
#pragma unroll
        for (int i = 0; i < kPerLane; ++i) {
            const int c = lane + 32 * i;
            if (c < chunks) {
                raw[i] = xr[c];
                if (rr) rraw[i] = rr[c];
            }
        }
    };
    load_row(row);
    for (; row < rows; row += warps_total) {
        float v[kPerLane][8];
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < kPerLane; ++i) {
            const int c = lane + 32 * i;
            if (c < chunks) {
                const uint32_t wa[4] = {raw[i].x, raw[i].y, raw[i].z, raw[i].w};
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    v[i][2 * u] = __uint_as_float(wa[u] << 16);
                    v[i][2 * u + 1] = __uint_as_float(wa[u] & 0xffff0000u);
                }
                if (res) {
                    const uint32_t wb[4] = {rraw[i].x, rraw[i].y, rraw[i].z, rraw[i].w};
                    uint32_t pk[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float s0 = v[i][2 * u] + __uint_as_float(wb[u] << 16);
                        const float s1 = v[i][2 * u + 1] + __uint_as_float(wb[u] & 0xffff0000u);
                        pk[u] = pack_bf16x2(s0, s1);
                        v[i][2 * u] = __uint_as_float(pk[u] << 16);  // the rounded sum is what is normalised
                        v[i][2 * u + 1] = __uint_as_float(pk[u] & 0xffff0000u);
                    }
                    if (sum_out)
                        reinterpret_cast<uint4 *>(sum_out + row * D)[c] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) sum += v[i][e];
            }
        }
        if (row + warps_total < rows) load_row(row + warps_total);  // in flight during the reductions
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float mean = sum / (float)D;
        float sq = 0.f;
#pragma unroll
        for (int i = 0; i < kPerLane; ++i)
            if (lane + 32 * i < chunks) {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float d = v[i][e] - mean;
                    sq = fmaf(d, d, sq);
                }
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        const float rstd = 1.f / sqrtf(sq / (float)D + eps);
        uint4 *yr = reinterpret_cast<uint4 *>(y + row * D);
#pragma unroll
        for (int i = 0; i < kPerLane; ++i) {
            const int c = lane + 32 * i;
            if (c < chunks) {
                uint32_t pk[4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    pk[u] = pack_bf16x2((v[i][2 * u] - mean) * rstd * g[i][2 * u] + bb[i][2 * u],
                                        (v[i][2 * u + 1] - mean) * rstd * g[i][2 * u + 1] + bb[i][2 * u + 1]);
                yr[c] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
        }
    }
}

}  // namespace gae
