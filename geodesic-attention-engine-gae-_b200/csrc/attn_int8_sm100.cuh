// attn_int8_sm100.cuh -- exact int32 QK^T logits on the tcgen05 int8 path.
//
// The int8 attention kernel (attn_sm100.cuh, int8 mode) consumes its logits
// from TMEM and never stores them.  This kernel runs the same tiles --
// TMA-loaded 128 x 128-byte int8 Q and K tiles in 128-byte swizzle, one
// tcgen05.mma kind::i8 per 32-byte K step, int32 accumulation in TMEM -- and
// writes them out, so the int8 arithmetic can be checked bit for bit against
// the reference's dot_int8 (cuda_src/waller_operator_int8.cu:13-24).
// CTA = one 128 x 128 logit tile of one (batch*head); 128 threads.
#pragma once
#include "sm100.cuh"

namespace gae {

struct Int8LogitsParams {
    CUtensorMap tm_q;  // dims {D, Nq, 1, BH}, box {128, 128, 1, 1}
    CUtensorMap tm_k;  // dims {D, Nkv, 1, BH}
    int32_t *out;      // [BH, Nq, Nkv]
    int Nq, Nkv;
};

enum Int8WaitSite : unsigned { kSiteLgLoad = 0x201, kSiteLgMma = 0x202 };

__global__ void __launch_bounds__(128) int8_logits_kernel(const __grid_constant__ Int8LogitsParams p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t base = (raw_addr + 1023u) & ~1023u;
    uint8_t *smem = smem_raw + (base - raw_addr);
    const uint32_t sQ = base, sK = base + 16384;
    const uint32_t bar_load = base + 32768, bar_mma = base + 32776;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + 32784);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + 32788);
    volatile int no_abort = 0;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * 128, n0 = blockIdx.y * 128, bh = blockIdx.z;

    if (threadIdx.x == 0) {
        mbar_init(bar_load, 1);
        mbar_init(bar_mma, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), 128);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    bool ok = true;
    if (threadIdx.x == 0) {
        mbar_expect_tx(bar_load, 32768);
        tma_load_4d(sQ, &p.tm_q, bar_load, 0, m0, 0, bh);
        tma_load_4d(sK, &p.tm_k, bar_load, 0, n0, 0, bh);
        ok = mbar_wait(bar_load, 0, kSiteLgLoad, &no_abort);
        if (ok) {
            constexpr uint32_t idesc = idesc_i8(128, 128);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                umma_i8_ss(tmem, smem_desc_sw128(sQ + kk * 32, 16, 1024),
                           smem_desc_sw128(sK + kk * 32, 16, 1024), idesc, kk > 0);
        }
        umma_commit(bar_mma);
    }
    __syncwarp();
    ok = mbar_wait(bar_mma, 0, kSiteLgMma, &no_abort);
    tc_fence_after();
    if (ok) {
        const int row = m0 + warp * 32 + lane;
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
        int32_t *orow = p.out + ((int64_t)bh * p.Nq + row) * p.Nkv;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            tmem_ld32(taddr + c * 32, r);
            tmem_wait_ld();
            if (row < p.Nq) {
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const int col = n0 + c * 32 + e;
                    if (col < p.Nkv) orow[col] = (int32_t)r[e];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, 128);
    }
}

}  // namespace gae
