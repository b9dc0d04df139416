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
// (causal: tiles i >= j only).  Per query tile the MMA warp issues
//   S = Q K^T, dP = dO V^T      (K-major x K-major)
//   dV += P^T dO                (P from shared memory read MN-major)
//   dK += dS^T Q                (dS likewise)
//   dQ  = dS K                  (dS K-major, K MN-major) into S's columns
// and the compute warpgroup turns S into P and dP into dS (bf16/f16 into
// shared memory in the 128-byte-swizzled layout both read directions share),
// then reads dQ out of TMEM and adds it to an fp32 accumulator in global
// memory with vector reductions (red.global.add.v4.f32): query tiles are
// shared by every key tile, so dQ is the one cross-CTA sum.
//
// Warps: 0-3 compute (thread = row of the 128-row tile, TMEM lane), 4 TMA,
// 5 MMA (owns TMEM).  TMEM columns: S / dQ [0,128), dP [128,256), dV
// [256,256+D), dK after it.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "sm100.cuh"

namespace gae {

struct AttnBwdParams {
    CUtensorMap tm_q, tm_k, tm_v, tm_do;  // dims {D, N, H, B}, box {64 elements, 128 rows}, 128B swizzle
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
};

template <int D>
struct AttnBwdCfg {
    static_assert(D == 64 || D == 128, "unsupported head_dim");
    static constexpr int kBox = 128 * 128;       // 128 rows x 128 bytes
    static constexpr int kPanels = D * 2 / 128;  // 64-element panels in a 128 x D tile
    static constexpr int kTile = kPanels * kBox;
    static constexpr int kPTile = 2 * kBox;      // 128 x 128, 16-bit
    static constexpr int kOffK = 0, kOffV = kTile, kOffQ = 2 * kTile, kOffDO = 3 * kTile;
    static constexpr int kOffP = 4 * kTile, kOffDS = kOffP + kPTile, kOffBar = kOffDS + kPTile;
    // kv, q_full, q_empty, s, dp, p, ds, dq, dq_free, done
    static constexpr int kNumBars = 10;
    static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;  // + alignment slack
    static constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256, kColDK = 256 + D;
    static constexpr uint32_t kTmemCols = 512;
    static constexpr int kThreads = 192;
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

__device__ __forceinline__ void red_add_v4(float *addr, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

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

template <int D, bool kBF16>
__global__ void __launch_bounds__(192, 1) attn_bwd_sm100_kernel(const __grid_constant__ AttnBwdParams p) {
    using Cfg = AttnBwdCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t *smem = smem_raw + (base - raw_addr);
    const uint32_t sK = base + Cfg::kOffK, sV = base + Cfg::kOffV, sQ = base + Cfg::kOffQ;
    const uint32_t sDO = base + Cfg::kOffDO, sP = base + Cfg::kOffP, sDS = base + Cfg::kOffDS;
    const uint32_t sBar = base + Cfg::kOffBar;
    const uint32_t bar_kv = sBar, bar_q_full = sBar + 8, bar_q_empty = sBar + 16, bar_s = sBar + 24;
    const uint32_t bar_dp = sBar + 32, bar_p = sBar + 40, bar_ds = sBar + 48, bar_dq = sBar + 56;
    const uint32_t bar_dq_free = sBar + 64, bar_done = sBar + 72;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + Cfg::kOffBar + Cfg::kNumBars * 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int no_abort = 0;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j = blockIdx.x, bh = blockIdx.y;
    const int b = bh / p.H, h = bh % p.H;
    const int n_q_tiles = (p.Nq + 127) / 128;
    const int i0 = p.causal ? j : 0;  // causal: Nq == Nkv and tile i sees key tile j only if i >= j
    const int n_it = n_q_tiles - i0;

    if (threadIdx.x == 0) {
        mbar_init(bar_kv, 1);
        mbar_init(bar_q_full, 1);
        mbar_init(bar_q_empty, 1);
        mbar_init(bar_s, 1);
        mbar_init(bar_dp, 1);
        mbar_init(bar_p, 128);
        mbar_init(bar_ds, 128);
        mbar_init(bar_dq, 1);
        mbar_init(bar_dq_free, 128);
        mbar_init(bar_done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 5) {
        tmem_alloc(smem_u32(tmem_slot), Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
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
            int issued = 0;
            for (int it = 0; it < n_it; ++it) {
                if (it > 0 && !mbar_wait(bar_q_empty, (it - 1) & 1, kSiteBwdQEmpty, abort_flag)) break;
                const int row0 = (i0 + it) * 128;
                mbar_expect_tx(bar_q_full, 2 * Cfg::kTile);
                for (int hf = 0; hf < Cfg::kPanels; ++hf) {
                    tma_load_4d(sQ + hf * Cfg::kBox, &p.tm_q, bar_q_full, hf * 64, row0, h, b);
                    tma_load_4d(sDO + hf * Cfg::kBox, &p.tm_do, bar_q_full, hf * 64, row0, h, b);
                }
                issued = it + 1;
            }
            // Drain: the copies issued have landed before the CTA exits.
            mbar_wait(bar_kv, 0, kSiteBwdKV, &no_abort);
            if (issued > 0) mbar_wait(bar_q_full, (issued - 1) & 1, kSiteBwdQFull, &no_abort);
        }
    } else if (warp == 5) {
        // ---------------------------------------------------------- MMA issuer
        if (lane == 0 && n_it > 0) {
            constexpr uint32_t id_qk = idesc_f16(128, 128, kBF16, false, false);
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
            bool ok = mbar_wait(bar_kv, 0, kSiteBwdKV, abort_flag);
            for (int it = 0; it < n_it && ok; ++it) {
                const uint32_t ph = it & 1;
                ok = mbar_wait(bar_q_full, ph, kSiteBwdQFull, abort_flag) &&
                     (it == 0 || mbar_wait(bar_dq_free, (it - 1) & 1, kSiteBwdDQFree, abort_flag));
                if (!ok) break;
                tc_fence_after();
                mma_kk(tmem + Cfg::kColS, sQ, sK);
                umma_commit(bar_s);
                mma_kk(tmem + Cfg::kColDP, sDO, sV);
                umma_commit(bar_dp);
                if (!(ok = mbar_wait(bar_p, ph, kSiteBwdP, abort_flag))) break;
                tc_fence_after();
                // dV += P^T dO: M = keys (MN-major in P), K = queries, N = D.
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    umma_f16_ss(tmem + Cfg::kColDV, smem_desc_sw128(sP + kk * 2048, Cfg::kBox, 1024),
                                smem_desc_sw128(sDO + kk * 2048, Cfg::kBox, 1024), id_t, (it > 0 || kk > 0));
                if (!(ok = mbar_wait(bar_ds, ph, kSiteBwdDS, abort_flag))) break;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    umma_f16_ss(tmem + Cfg::kColDK, smem_desc_sw128(sDS + kk * 2048, Cfg::kBox, 1024),
                                smem_desc_sw128(sQ + kk * 2048, Cfg::kBox, 1024), id_t, (it > 0 || kk > 0));
                // dQ = dS K: M = queries, K = keys (K-major in dS), N = D (MN-major in K).
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t off = (kk >> 2) * Cfg::kBox + (kk & 3) * 32;
                    umma_f16_ss(tmem + Cfg::kColS, smem_desc_sw128(sDS + off, 16, 1024),
                                smem_desc_sw128(sK + kk * 2048, Cfg::kBox, 1024), id_dq, kk > 0);
                }
                umma_commit(bar_dq);
                umma_commit(bar_q_empty);
            }
            umma_commit(bar_done);
            mbar_wait(bar_done, 0, kSiteBwdDone, &no_abort);
        }
    } else {
        // ------------------------------------------------ compute warpgroup
        const int row = warp * 32 + lane;
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        const uint32_t tS = tmem + lane_off + Cfg::kColS, tDP = tmem + lane_off + Cfg::kColDP;
        bool ok = n_it > 0;
        for (int it = 0; it < n_it && ok; ++it) {
            const uint32_t ph = it & 1;
            const int q = (i0 + it) * 128 + row;
            const bool valid = q < p.Nq;
            float lse2 = INFINITY, dlt = 0.f;  // +inf: the row contributes nothing
            if (valid) {
                const float l = p.lse[(int64_t)bh * p.Nq + q];
                if (l != -INFINITY) lse2 = l * 1.4426950408889634f;
                dlt = p.delta[(int64_t)bh * p.Nq + q];
            }
            // Keys of this tile this row may see: [0, lim).
            int lim = min(128, p.Nkv - j * 128);
            if (p.causal) lim = min(lim, max(0, q - j * 128 + 1));

            if (!(ok = mbar_wait(bar_s, ph, kSiteBwdS, abort_flag))) break;
            tc_fence_after();
            uint32_t pk[64];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t r[32];
                tmem_ld32(tS + c * 32, r);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const int k0 = c * 32 + 2 * e;
                    const float p0 = (k0 < lim) ? ex2_approx(__uint_as_float(r[2 * e]) * p.scale_log2 - lse2) : 0.f;
                    const float p1 =
                        (k0 + 1 < lim) ? ex2_approx(__uint_as_float(r[2 * e + 1]) * p.scale_log2 - lse2) : 0.f;
                    pk[c * 16 + e] = kBF16 ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
                }
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    st_shared_v4(sP + sw128_chunk(row, c * 4 + u), pk[c * 16 + 4 * u], pk[c * 16 + 4 * u + 1],
                                 pk[c * 16 + 4 * u + 2], pk[c * 16 + 4 * u + 3]);
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(bar_p);

            if (!(ok = mbar_wait(bar_dp, ph, kSiteBwdDP, abort_flag))) break;
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t r[32], dk[16];
                tmem_ld32(tDP + c * 32, r);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    float p0, p1;
                    unpack2<kBF16>(pk[c * 16 + e], p0, p1);
                    const float d0 = p0 * (__uint_as_float(r[2 * e]) - dlt);
                    const float d1 = p1 * (__uint_as_float(r[2 * e + 1]) - dlt);
                    dk[e] = kBF16 ? pack_bf16x2(d0, d1) : pack_f16x2(d0, d1);
                }
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    st_shared_v4(sDS + sw128_chunk(row, c * 4 + u), dk[4 * u], dk[4 * u + 1], dk[4 * u + 2],
                                 dk[4 * u + 3]);
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(bar_ds);

            if (!(ok = mbar_wait(bar_dq, ph, kSiteBwdDQ, abort_flag))) break;
            tc_fence_after();
            float *dq_row = p.dq_acc + ((int64_t)bh * p.Nq + (valid ? q : 0)) * D;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(tS + c * 32, r);
                tmem_wait_ld();
                if (valid) {
#pragma unroll
                    for (int v = 0; v < 8; ++v)
                        red_add_v4(dq_row + c * 32 + 4 * v, __uint_as_float(r[4 * v]) * p.scale,
                                   __uint_as_float(r[4 * v + 1]) * p.scale, __uint_as_float(r[4 * v + 2]) * p.scale,
                                   __uint_as_float(r[4 * v + 3]) * p.scale);
                }
            }
            tc_fence_before();
            mbar_arrive(bar_dq_free);
        }
        // Epilogue: dV and scale * dK of this key tile -> global.
        if (ok && mbar_wait(bar_done, 0, kSiteBwdDone, abort_flag)) {
            tc_fence_after();
            const int key = j * 128 + row;
            const bool kvalid = key < p.Nkv;
            for (int t = 0; t < 2; ++t) {
                const uint32_t tc = tmem + lane_off + (t ? Cfg::kColDK : Cfg::kColDV);
                const float mul = t ? p.scale : 1.f;
                char *dst = reinterpret_cast<char *>(t ? p.dk : p.dv) +
                            2 * (t ? (b * p.dk_sb + h * p.dk_sh + (int64_t)key * p.dk_ss)
                                   : (b * p.dv_sb + h * p.dv_sh + (int64_t)key * p.dv_ss));
#pragma unroll
                for (int c = 0; c < D / 32; ++c) {
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
    if (warp == 5) {
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
