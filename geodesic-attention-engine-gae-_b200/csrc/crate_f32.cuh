// crate_f32.cuh -- fp32 kernels for the reference crate's layer functions,
// computed in the crate's own operation order.
//
// The crate (rust_src/src/layernorm.rs, mlp.rs, transformer.rs) computes in
// f32 with one accumulator per output and a strictly sequential sum.  These
// kernels keep exactly that order per output element (one thread owns an
// output's accumulator and walks the reduction index upward) and use explicit
// round-to-nearest intrinsics so that no multiply-add is contracted; the
// results are then bit-identical to the crate's for the sums, LayerNorm
// statistics and normalisation.  GELU goes through tanhf, whose last-place
// rounding may differ from the host libm's.
//
// Work is spread over many outputs at once (the GPU's parallelism is across
// tokens and output features, never inside one sum).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace gae {

// rust_src/src/activations.rs:5-7: 0.5*x*(1 + tanh(sqrt(2/pi)*(x + 0.044715*x^3)))
// with x.powi(3) = (x*x)*x and sqrt(2/pi) the f32 root of the f32 quotient.
__device__ __forceinline__ float crate_gelu(float x) {
    const float c = sqrtf(2.0f / 3.14159265358979323846f);
    const float x3 = __fmul_rn(__fmul_rn(x, x), x);
    const float inner = __fmul_rn(c, __fadd_rn(x, __fmul_rn(0.044715f, x3)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

// Y[t, n] = epi(init_n + sum_{j=0..K-1} x[t, j] * W(j, n)), the sum taken in
// increasing j, init_n = bias[n] (mlp.rs:17-22, 26-31) or 0 (the matvec of
// transformer.rs:124-134).  W(j, n) = w[j*N + n] when kWInMajor (the crate's
// W1 [hidden, mlp], W2 [mlp, hidden]) else w[n*K + j] (W[out, in], the
// crate's wq/wk/wv/wo).  epi: 0 none, 1 GELU, 2 + res[t, n] after the sum
// (the crate's residual add of the finished output).
//
// 256 threads, a 64-token x 64-output tile, each thread 4 x 4 outputs whose
// accumulators all step through j together; x and W staged 16 j at a time
// in shared memory.
constexpr int kCrateBM = 64, kCrateBN = 64, kCrateBK = 16;

template <bool kWInMajor>
__global__ void __launch_bounds__(256) crate_linear_f32_kernel(
    const float *__restrict__ x, const float *__restrict__ w, const float *__restrict__ bias,
    const float *__restrict__ res, float *__restrict__ y, int64_t M, int64_t N, int64_t K, int epi) {
    __shared__ float xs[kCrateBK][kCrateBM + 4];
    __shared__ float ws[kCrateBK][kCrateBN + 4];
    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;           // outputs tx*4.., tokens ty*4..
    const int64_t m0 = (int64_t)blockIdx.y * kCrateBM, n0 = (int64_t)blockIdx.x * kCrateBN;

    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int64_t n = n0 + tx * 4 + j;
        const float init = (bias != nullptr && n < N) ? bias[n] : 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i][j] = init;
    }

    for (int64_t k0 = 0; k0 < K; k0 += kCrateBK) {
        const int kn = (int)((K - k0) < kCrateBK ? (K - k0) : kCrateBK);
        // x tile [64 tokens][16 j] -> xs[j][token]; 1024 values, 4 per thread
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int idx = tid + r * 256;
            const int kk = idx % kCrateBK, mm = idx / kCrateBK;
            const int64_t m = m0 + mm, k = k0 + kk;
            xs[kk][mm] = (m < M && kk < kn) ? x[m * K + k] : 0.0f;
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int idx = tid + r * 256;
            int kk, nn;
            if (kWInMajor) { nn = idx % kCrateBN; kk = idx / kCrateBN; }   // rows of W are j
            else { kk = idx % kCrateBK; nn = idx / kCrateBK; }              // rows of W are n
            const int64_t n = n0 + nn, k = k0 + kk;
            float v = 0.0f;
            if (n < N && kk < kn) v = kWInMajor ? w[k * N + n] : w[n * K + k];
            ws[kk][nn] = v;
        }
        __syncthreads();
        for (int kk = 0; kk < kn; ++kk) {  // only real j: no +0 terms enter a sum
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = xs[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = ws[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
        }
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t m = m0 + ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t n = n0 + tx * 4 + j;
            if (n >= N) continue;
            float v = acc[i][j];
            if (epi == 1) v = crate_gelu(v);
            else if (epi == 2) v = __fadd_rn(v, res[m * N + n]);
            y[m * N + n] = v;
        }
    }
}

// Row LayerNorm with the crate's single-pass Welford statistics
// (rust_src/src/welford.rs:27-43, layernorm.rs:6-47): per row, in order,
// count += 1; delta = x - mean; mean += delta/count; m2 += delta*(x - mean);
// std = sqrt(m2/count + eps) (variance 0 below two samples);
// y = (x - mean)/std*gamma + beta.
// One warp per 32 rows: 32 x 32 tiles are read coalesced into shared memory
// and each lane then walks its own row's 32 values in order; the normalising
// pass is coalesced over columns.
__global__ void __launch_bounds__(128) crate_layernorm_f32_kernel(
    const float *__restrict__ x, const float *__restrict__ gamma, const float *__restrict__ beta,
    float *__restrict__ y, int64_t rows, int64_t d, float eps) {
    __shared__ float tile[4][32][33];
    __shared__ float stat[4][32][2];
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int64_t r0 = ((int64_t)blockIdx.x * 4 + warp) * 32;
    if (r0 >= rows) return;
    const int nr = (int)((rows - r0) < 32 ? (rows - r0) : 32);
    float mean = 0.0f, m2 = 0.0f;
    uint32_t count = 0;
    for (int64_t c0 = 0; c0 < d; c0 += 32) {
        const int nc = (int)((d - c0) < 32 ? (d - c0) : 32);
        for (int r = 0; r < nr; ++r)
            if (lane < nc) tile[warp][r][lane] = x[(r0 + r) * d + c0 + lane];
        __syncwarp();
        if (lane < nr) {
            for (int c = 0; c < nc; ++c) {
                const float v = tile[warp][lane][c];
                count += 1;
                const float delta = __fsub_rn(v, mean);
                mean = __fadd_rn(mean, __fdiv_rn(delta, (float)count));
                const float delta2 = __fsub_rn(v, mean);
                m2 = __fadd_rn(m2, __fmul_rn(delta, delta2));
            }
        }
        __syncwarp();
    }
    if (lane < nr) {
        const float var = count < 2 ? 0.0f : __fdiv_rn(m2, (float)count);
        stat[warp][lane][0] = mean;
        stat[warp][lane][1] = __fsqrt_rn(__fadd_rn(var, eps));
    }
    __syncwarp();
    for (int r = 0; r < nr; ++r) {
        const float mu = stat[warp][r][0], sd = stat[warp][r][1];
        const float *xr = x + (r0 + r) * d;
        float *yr = y + (r0 + r) * d;
        for (int64_t c = lane; c < d; c += 32)
            yr[c] = __fadd_rn(__fmul_rn(__fdiv_rn(__fsub_rn(xr[c], mu), sd), gamma[c]), beta[c]);
    }
}

}  // namespace gae
