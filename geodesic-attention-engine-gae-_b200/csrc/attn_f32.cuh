// attn_f32.cuh -- fp32 exact attention on the CUDA cores: the parity path for
// the reference's fp32 Waller operator (rust_src/src/waller_operator.rs:8-59;
// GPU behaviour cuda_src/waller_operator.cu:12-100).
//
// One thread owns one query row and runs the reference's per-key recurrence
// in the reference's operation order: sequential dot product then * scale,
// the branchy OnlineSoftmax update (online_softmax.rs:28-35), the correction
// exp(old_max - max) applied when old_max != -inf, acc += exp(score - max) * v,
// and a final division by the sum.  Every multiply and add is an explicit
// round-to-nearest operation (no FMA contraction), so the result differs from
// the Rust path only by the exp implementation.  K/V tiles of 32 keys are
// staged in shared memory and shared by the 128 rows of a block; the query
// rows live in shared memory transposed ([c][row]) so that the per-thread
// reads are conflict-free and the K/V reads are broadcasts.
#pragma once
#include "sm100.cuh"

namespace gae {

struct AttnF32Params {
    const float *q, *k, *v;
    float *o;
    float *lse;
    int64_t q_sb, q_sh, q_ss, k_sb, k_sh, k_ss, v_sb, v_sh, v_ss, o_sb, o_sh, o_ss;
    int B, H, Nq, Nkv, D;
    int causal;
    float scale;
    int64_t q_offset, kv_offset;
};

constexpr int kF32Rows = 128;
constexpr int kF32Keys = 32;

template <int DMAX>
__global__ void __launch_bounds__(kF32Rows) attn_fwd_f32_kernel(const AttnF32Params p) {
    extern __shared__ float smf[];
    float *q_s = smf;                          // [DMAX][kF32Rows]
    float *k_s = q_s + DMAX * kF32Rows;        // [kF32Keys][DMAX]
    float *v_s = k_s + kF32Keys * DMAX;        // [kF32Keys][DMAX]

    const int tid = threadIdx.x;
    const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
    const int r0 = blockIdx.x * kF32Rows;
    const int row = r0 + tid;
    const int D = p.D;
    const bool valid = row < p.Nq;
    const float *qb = p.q + b * p.q_sb + h * p.q_sh;
    const float *kb = p.k + b * p.k_sb + h * p.k_sh;
    const float *vb = p.v + b * p.v_sb + h * p.v_sh;

    // Stage this block's query rows, transposed.
    for (int idx = tid; idx < kF32Rows * D; idx += kF32Rows) {
        const int rr = idx / D, c = idx % D;
        const int qr = r0 + rr;
        q_s[c * kF32Rows + rr] = (qr < p.Nq) ? qb[(int64_t)qr * p.q_ss + c] : 0.f;
    }

    // Keys visible to this thread: [0, jend).
    int64_t jend = p.Nkv;
    int64_t block_end = p.Nkv;
    if (p.causal) {
        jend = min64(jend, max64(0, p.q_offset + row - p.kv_offset + 1));
        const int last_row = min(r0 + kF32Rows - 1, p.Nq - 1);
        block_end = min64(block_end, max64(0, p.q_offset + last_row - p.kv_offset + 1));
    }

    float acc[DMAX];
#pragma unroll
    for (int c = 0; c < DMAX; ++c) acc[c] = 0.f;
    float m = -INFINITY, l = 0.f;

    for (int64_t t0 = 0; t0 < block_end; t0 += kF32Keys) {
        __syncthreads();
        const int nk = (int)min64(kF32Keys, block_end - t0);
        for (int idx = tid; idx < nk * D; idx += kF32Rows) {
            const int kr = idx / D, c = idx % D;
            k_s[kr * DMAX + c] = kb[(t0 + kr) * p.k_ss + c];
            v_s[kr * DMAX + c] = vb[(t0 + kr) * p.v_ss + c];
        }
        __syncthreads();
        if (!valid) continue;
        const int my_n = (int)max64(0, min64(nk, jend - t0));
        for (int j = 0; j < my_n; ++j) {
            float dot = 0.f;
#pragma unroll
            for (int c = 0; c < DMAX; ++c)
                if (c < D) dot = __fadd_rn(dot, __fmul_rn(q_s[c * kF32Rows + tid], k_s[j * DMAX + c]));
            const float score = __fmul_rn(dot, p.scale);
            const float old_m = m;
            if (score > m) {
                l = __fadd_rn(__fmul_rn(l, expf(__fsub_rn(m, score))), 1.f);
                m = score;
            } else {
                l = __fadd_rn(l, expf(__fsub_rn(score, m)));
            }
            if (old_m != -INFINITY) {
                const float corr = expf(__fsub_rn(old_m, m));
#pragma unroll
                for (int c = 0; c < DMAX; ++c) acc[c] = __fmul_rn(acc[c], corr);
            }
            const float w = expf(__fsub_rn(score, m));
#pragma unroll
            for (int c = 0; c < DMAX; ++c)
                if (c < D) acc[c] = __fadd_rn(acc[c], __fmul_rn(w, v_s[j * DMAX + c]));
        }
    }
    if (!valid) return;
    float *orow = p.o + b * p.o_sb + h * p.o_sh + (int64_t)row * p.o_ss;
    if (jend <= 0) {
        for (int c = 0; c < D; ++c) orow[c] = 0.f;
        if (p.lse) p.lse[(int64_t)bh * p.Nq + row] = -INFINITY;
        return;
    }
#pragma unroll
    for (int c = 0; c < DMAX; ++c)
        if (c < D) orow[c] = __fdiv_rn(acc[c], l);
    if (p.lse) p.lse[(int64_t)bh * p.Nq + row] = __fadd_rn(m, logf(l));
}

// ------------------------------------------------------------ LSE merge
// One warp per row.  o_acc = (a*o_acc + b*o_part)/(a+b), lse_acc = m+log(a+b)
// with m = max(lse_acc, lse_part), a = e^(lse_acc-m), b = e^(lse_part-m).
template <typename T>
__device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <typename T>
__device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

template <typename TA, typename TP>
__global__ void lse_merge_kernel(TA *o_acc, float *lse_acc, const TP *o_part, const float *lse_part,
                                 int64_t rows, int D, int64_t sa, int64_t sp) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float la = lse_acc[row], lb = lse_part[row];
    const float mx = fmaxf(la, lb);
    if (mx == -INFINITY) return;
    const float wa = expf(la - mx), wb = expf(lb - mx);
    const float s = wa + wb;
    TA *oa = o_acc + row * sa;
    const TP *op = o_part + row * sp;
    for (int c = lane; c < D; c += 32)
        oa[c] = from_f<TA>((wa * to_f<TA>(oa[c]) + wb * to_f<TP>(op[c])) / s);
    if (lane == 0) lse_acc[row] = mx + logf(s);
}

// ---------------------------------------------------- int8 quantisation
// One warp per row: scale = max|x| / 127, q = rint(x / scale) clamped.
template <typename T>
__global__ void quantize_rows_int8_kernel(const T *x, int64_t rows, int D, int8_t *q, float *scale) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const T *xr = x + row * D;
    float mx = 0.f;
    for (int c = lane; c < D; c += 32) mx = fmaxf(mx, fabsf(to_f<T>(xr[c])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float s = __fdiv_rn(mx, 127.f);
    for (int c = lane; c < D; c += 32) {
        float v = (s > 0.f) ? rintf(__fdiv_rn(to_f<T>(xr[c]), s)) : 0.f;
        v = fminf(fmaxf(v, -127.f), 127.f);
        q[row * D + c] = (int8_t)v;
    }
    if (lane == 0) scale[row] = s;
}

}  // namespace gae
