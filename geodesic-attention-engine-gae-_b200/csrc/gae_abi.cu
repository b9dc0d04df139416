// gae_abi.cu -- the C ABI of libgae.so (declared in include/gae.h).
//
// This translation unit owns argument validation, error reporting, TMA
// descriptor encoding and kernel launches.  The kernels live in the headers
// it includes (one translation unit, so that the device-side error record
// gae_dev_error is a single symbol without relocatable device code).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/gae.h"
#include "../../include/gae_debug.h"
#include "attn_f32.cuh"
#include "attn_sm100.cuh"
#include "attn_bwd_sm100.cuh"
#include "attn_int8_sm100.cuh"
#include "layer_sm100.cuh"
#include "symphony.cuh"
#include "crate_f32.cuh"

namespace {

thread_local char g_err[512] = "";
thread_local gae_status g_err_status = GAE_OK;

gae_status fail(gae_status s, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    g_err_status = s;
    return s;
}

#define GAE_CUDA_TRY(expr)                                                                 \
    do {                                                                                   \
        cudaError_t e_ = (expr);                                                           \
        if (e_ != cudaSuccess)                                                             \
            return fail(e_ == cudaErrorMemoryAllocation ? GAE_ERR_OOM : GAE_ERR_CUDA,     \
                        "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, \
                        __LINE__);                                                         \
    } while (0)

// ---------------------------------------------------------------- TMA maps
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 4-D map over a [B, H, N, D] view with element strides {sb, sh, ss, 1},
// box {64 elements (128 B), box_rows, 1, 1}, 128-byte swizzle.
gae_status make_map_4d(CUtensorMap *m, const void *ptr, CUtensorMapDataType dt, int esize,
                       int64_t B, int64_t H, int64_t N, int64_t D, int64_t sb, int64_t sh,
                       int64_t ss, int box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(GAE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)N, (cuuint64_t)H, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)(ss * esize), (cuuint64_t)(sh * esize),
                             (cuuint64_t)(sb * esize)};
    cuuint32_t box[4] = {(cuuint32_t)(128 / esize), (cuuint32_t)box_rows, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, dt, 4, const_cast<void *>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GAE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return GAE_OK;
}

int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename Kern>
gae_status set_smem(Kern k, int bytes) {
    GAE_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    return GAE_OK;
}

// 2-D fp32 map over a [rows, n] row-major array, box {128, 1}, no swizzle
// (the per-key int8 dequantisation scales).
gae_status make_map_2d_f32(CUtensorMap *m, const void *ptr, int64_t n, int64_t rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(GAE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    if ((n * 4) % 16 != 0)
        return fail(GAE_ERR_INVALID_ARG, "int8 attention needs seq %% 4 == 0 (16-byte scale rows)");
    cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(n * 4)};
    cuuint32_t box[2] = {128, 1};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(ptr), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GAE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return GAE_OK;
}

template <int D, int kMode, bool kDump = false>
gae_status launch_tc(const gae::AttnParams &p, dim3 grid, cudaStream_t st) {
    auto kern = gae::attn_fwd_sm100_kernel<D, kMode, kDump>;
    constexpr int smem = gae::AttnCfg<D, kMode>::kSmemBytes;
    gae_status s = set_smem(kern, smem);
    if (s != GAE_OK) return s;
    kern<<<grid, gae::AttnCfg<D, kMode>::kThreads, smem, st>>>(p);
    GAE_CUDA_TRY(cudaGetLastError());
    return GAE_OK;
}

// ------------------------------------------------------------ attention
gae_status launch_attn_tc(const gae_attn_args *a, cudaStream_t st) {
    const bool bf16 = a->dtype == GAE_DTYPE_BF16;
    const int64_t D = a->head_dim;
    if (D != 64 && D != 128)
        return fail(GAE_ERR_UNSUPPORTED, "tensor-core attention supports head_dim 64 or 128, got %lld",
                    (long long)D);
    const void *ptrs[4] = {a->q, a->k, a->v, a->o};
    for (const void *pp : ptrs)
        if (!aligned16(pp)) return fail(GAE_ERR_INVALID_ARG, "q/k/v/o must be 16-byte aligned");
    const int64_t *strs[4] = {a->q_stride, a->k_stride, a->v_stride, a->o_stride};
    for (const int64_t *s : strs)
        for (int i = 0; i < 3; ++i)
            if (s[i] < 0 || (s[i] % 8) != 0)
                return fail(GAE_ERR_INVALID_ARG,
                            "strides must be non-negative multiples of 8 elements (16 bytes)");
    if (a->batch * a->heads > 65535) return fail(GAE_ERR_UNSUPPORTED, "batch*heads > 65535");
    if (a->seq_q > (1ll << 30) || a->seq_kv > (1ll << 30))
        return fail(GAE_ERR_UNSUPPORTED, "sequence longer than 2^30");
    if (!(a->scale >= 0.f))
        return fail(GAE_ERR_UNSUPPORTED, "tensor-core attention needs a non-negative scale");

    gae::AttnParams p;
    memset(&p, 0, sizeof(p));
    const CUtensorMapDataType dt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    gae_status s;
    if ((s = make_map_4d(&p.tm_q, a->q, dt, 2, a->batch, a->heads, a->seq_q, D, a->q_stride[0],
                         a->q_stride[1], a->q_stride[2], 128)) != GAE_OK)
        return s;
    if ((s = make_map_4d(&p.tm_k, a->k, dt, 2, a->batch, a->heads, a->seq_kv, D, a->k_stride[0],
                         a->k_stride[1], a->k_stride[2], 128)) != GAE_OK)
        return s;
    if ((s = make_map_4d(&p.tm_v, a->v, dt, 2, a->batch, a->heads, a->seq_kv, D, a->v_stride[0],
                         a->v_stride[1], a->v_stride[2], 128)) != GAE_OK)
        return s;
    p.o = a->o;
    p.lse = a->lse;
    p.o_sb = a->o_stride[0];
    p.o_sh = a->o_stride[1];
    p.o_ss = a->o_stride[2];
    p.B = (int)a->batch;
    p.H = (int)a->heads;
    p.Nq = (int)a->seq_q;
    p.Nkv = (int)a->seq_kv;
    p.n_qpairs = (int)((a->seq_q + 255) / 256);
    p.causal = a->causal ? 1 : 0;
    p.scale_log2 = a->scale * 1.4426950408889634f;
    p.q_offset = a->q_offset;
    p.kv_offset = a->kv_offset;
    const int64_t units = (int64_t)p.n_qpairs * a->batch * a->heads;
    if (units > (1ll << 30)) return fail(GAE_ERR_UNSUPPORTED, "too many query blocks");
    // head_dim 64: one persistent CTA per SM walks the units (its short units
    // gain most from keeping TMEM, barriers and the K/V stream alive, measured
    // +20%).  head_dim 128: one CTA per unit, balanced by the hardware's block
    // scheduler (equal or better under the power cap, measured).
    // head_dim 128 stays one CTA per unit, causal and not: a persistent
    // head-major grid gave config 2 non-causal +1.5% (1284 vs 1267) alone,
    // but the two-GPU ring, whose off-diagonal steps are non-causal, ran at
    // 2220 against 2256 with it (power-capped, NCCL's kernels beside it).
    bool persistent = D == 64 && units > num_sms();
    p.head_major = persistent ? 0 : 1;
    {
        // Diagnostics overrides of the schedule: GAE_ATTN_PERSISTENT=0/1 and
        // GAE_ATTN_HEAD_MAJOR=0/1 (unit order of the persistent grid).
        static const char *env_p = getenv("GAE_ATTN_PERSISTENT");
        static const char *env_h = getenv("GAE_ATTN_HEAD_MAJOR");
        if (env_p && (env_p[0] == '0' || env_p[0] == '1')) {
            persistent = env_p[0] == '1' && units > num_sms();
            p.head_major = persistent ? 0 : 1;
        }
        if (persistent && env_h && (env_h[0] == '0' || env_h[0] == '1')) p.head_major = env_h[0] - '0';
    }
    dim3 grid((unsigned)(persistent ? num_sms() : units));

    if (D == 128) {
        if (bf16) s = launch_tc<128, gae::kModeBF16>(p, grid, st);
        else s = launch_tc<128, gae::kModeF16>(p, grid, st);
    } else {
        if (bf16) s = launch_tc<64, gae::kModeBF16>(p, grid, st);
        else s = launch_tc<64, gae::kModeF16>(p, grid, st);
    }
    return s;
}

size_t attn_bwd_ws_region(int64_t B, int64_t H, int64_t N, int64_t D) {
    return ((size_t)(B * H * N * D) * 4 + 255) & ~(size_t)255;
}

template <int D, bool kBF16>
gae_status launch_bwd_tc(const gae::AttnBwdParams &p, dim3 grid, cudaStream_t st) {
    auto kern = gae::attn_bwd_sm100_kernel<D, kBF16>;
    constexpr int smem = gae::AttnBwdCfg<D>::kSmemBytes;
    gae_status s = set_smem(kern, smem);
    if (s != GAE_OK) return s;
    kern<<<grid, gae::AttnBwdCfg<D>::kThreads, smem, st>>>(p);
    GAE_CUDA_TRY(cudaGetLastError());
    return GAE_OK;
}

gae_status launch_attn_bwd(const gae_attn_bwd_args *a, cudaStream_t st) {
    const int64_t B = a->batch, H = a->heads, Nq = a->seq_q, Nkv = a->seq_kv, D = a->head_dim;
    if (B < 1 || H < 1 || Nq < 1 || Nkv < 1) return fail(GAE_ERR_INVALID_ARG, "empty or negative shape");
    if (D != 64 && D != 128)
        return fail(GAE_ERR_UNSUPPORTED, "attention backward supports head_dim 64 or 128, got %lld", (long long)D);
    if (a->dtype != GAE_DTYPE_BF16 && a->dtype != GAE_DTYPE_F16)
        return fail(GAE_ERR_UNSUPPORTED, "attention backward supports bf16 and f16");
    if (a->causal && Nq != Nkv) return fail(GAE_ERR_UNSUPPORTED, "causal backward needs seq_q == seq_kv");
    if (B * H > 65535) return fail(GAE_ERR_UNSUPPORTED, "batch*heads > 65535");
    if (Nq > (1ll << 30) || Nkv > (1ll << 30)) return fail(GAE_ERR_UNSUPPORTED, "sequence longer than 2^30");
    if (!(a->scale >= 0.f)) return fail(GAE_ERR_UNSUPPORTED, "negative or NaN scale");
    const void *ptrs[10] = {a->q, a->k, a->v, a->o, a->dout, a->lse, a->dq, a->dk, a->dv, a->workspace};
    for (const void *pp : ptrs)
        if (!pp) return fail(GAE_ERR_INVALID_ARG, "NULL pointer in attention backward arguments");
        else if (!aligned16(pp)) return fail(GAE_ERR_INVALID_ARG, "attention backward pointers must be 16-byte aligned");
    const int64_t *strs[8] = {a->q_stride, a->k_stride, a->v_stride, a->o_stride,
                              a->do_stride, a->dq_stride, a->dk_stride, a->dv_stride};
    for (const int64_t *sp : strs)
        for (int i = 0; i < 3; ++i)
            if (sp[i] < 0 || (sp[i] % 8) != 0)
                return fail(GAE_ERR_INVALID_ARG, "strides must be non-negative multiples of 8 elements");
    const size_t need = gae_attn_bwd_workspace_bytes(B, H, Nq, D);
    if (a->workspace_bytes < need)
        return fail(GAE_ERR_INVALID_ARG, "workspace too small: %zu < %zu", a->workspace_bytes, need);

    const bool bf16 = a->dtype == GAE_DTYPE_BF16;
    float *dq_acc = static_cast<float *>(a->workspace);
    float *delta = reinterpret_cast<float *>(static_cast<char *>(a->workspace) + attn_bwd_ws_region(B, H, Nq, D));
    GAE_CUDA_TRY(cudaMemsetAsync(dq_acc, 0, (size_t)(B * H * Nq * D) * 4, st));
    {
        const int64_t rows = B * H * Nq;
        const unsigned blocks = (unsigned)((rows + 7) / 8);
        if (bf16)
            gae::attn_bwd_delta_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
                (const __nv_bfloat16 *)a->o, (const __nv_bfloat16 *)a->dout, delta, (int)B, (int)H, (int)Nq, (int)D,
                a->o_stride[0], a->o_stride[1], a->o_stride[2], a->do_stride[0], a->do_stride[1], a->do_stride[2]);
        else
            gae::attn_bwd_delta_kernel<__half><<<blocks, 256, 0, st>>>(
                (const __half *)a->o, (const __half *)a->dout, delta, (int)B, (int)H, (int)Nq, (int)D,
                a->o_stride[0], a->o_stride[1], a->o_stride[2], a->do_stride[0], a->do_stride[1], a->do_stride[2]);
        GAE_CUDA_TRY(cudaGetLastError());
    }
    gae::AttnBwdParams p;
    memset(&p, 0, sizeof(p));
    const CUtensorMapDataType dt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    gae_status s;
    if ((s = make_map_4d(&p.tm_q, a->q, dt, 2, B, H, Nq, D, a->q_stride[0], a->q_stride[1], a->q_stride[2], 128)) ||
        (s = make_map_4d(&p.tm_k, a->k, dt, 2, B, H, Nkv, D, a->k_stride[0], a->k_stride[1], a->k_stride[2], 128)) ||
        (s = make_map_4d(&p.tm_v, a->v, dt, 2, B, H, Nkv, D, a->v_stride[0], a->v_stride[1], a->v_stride[2], 128)) ||
        (s = make_map_4d(&p.tm_do, a->dout, dt, 2, B, H, Nq, D, a->do_stride[0], a->do_stride[1], a->do_stride[2],
                         128)))
        return s;
    {
        // fp32 dQ accumulator [B*H, Nq, D]: 3-D map so that a tile's rows past
        // Nq (the ragged end of a head) fall outside the tensor and are skipped.
        EncodeTiledFn enc = encode_fn();
        if (!enc) return fail(GAE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
        cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)Nq, (cuuint64_t)(B * H)};
        cuuint64_t strides[2] = {(cuuint64_t)(D * 4), (cuuint64_t)(Nq * D * 4)};
        cuuint32_t box[3] = {32, 128, 1};
        cuuint32_t estr[3] = {1, 1, 1};
        CUresult r = enc(&p.tm_dq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, dq_acc, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) return fail(GAE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    }
    p.lse = a->lse;
    p.delta = delta;
    p.dq_acc = dq_acc;
    p.dk = a->dk;
    p.dv = a->dv;
    p.dk_sb = a->dk_stride[0]; p.dk_sh = a->dk_stride[1]; p.dk_ss = a->dk_stride[2];
    p.dv_sb = a->dv_stride[0]; p.dv_sh = a->dv_stride[1]; p.dv_ss = a->dv_stride[2];
    p.B = (int)B; p.H = (int)H; p.Nq = (int)Nq; p.Nkv = (int)Nkv;
    p.causal = a->causal ? 1 : 0;
    p.scale = a->scale;
    p.scale_log2 = a->scale * 1.4426950408889634f;
    dim3 grid((unsigned)((Nkv + 127) / 128), (unsigned)(B * H));
    if (D == 128) s = bf16 ? launch_bwd_tc<128, true>(p, grid, st) : launch_bwd_tc<128, false>(p, grid, st);
    else s = bf16 ? launch_bwd_tc<64, true>(p, grid, st) : launch_bwd_tc<64, false>(p, grid, st);
    if (s != GAE_OK) return s;
    {
        const int64_t total4 = B * H * Nq * D / 4;
        const unsigned blocks = (unsigned)((total4 + 255) / 256);
        if (bf16)
            gae::attn_bwd_dq_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
                dq_acc, (__nv_bfloat16 *)a->dq, (int)B, (int)H, (int)Nq, (int)D, a->dq_stride[0], a->dq_stride[1],
                a->dq_stride[2]);
        else
            gae::attn_bwd_dq_kernel<__half><<<blocks, 256, 0, st>>>(dq_acc, (__half *)a->dq, (int)B, (int)H,
                                                                      (int)Nq, (int)D, a->dq_stride[0],
                                                                      a->dq_stride[1], a->dq_stride[2]);
        GAE_CUDA_TRY(cudaGetLastError());
    }
    return GAE_OK;
}

gae_status launch_attn_int8(const gae_attn_int8_args *a, cudaStream_t st, int32_t *logits_dump = nullptr) {
    const int64_t D = a->head_dim, BH = a->batch_heads, N = a->seq;
    if (D != 128) return fail(GAE_ERR_UNSUPPORTED, "int8 attention supports head_dim 128, got %lld", (long long)D);
    if (BH > 65535) return fail(GAE_ERR_UNSUPPORTED, "batch_heads > 65535");
    if (N > (1ll << 30)) return fail(GAE_ERR_UNSUPPORTED, "sequence longer than 2^30");
    const void *ptrs[6] = {a->q, a->k, a->q_scale, a->k_scale, a->v, a->o};
    for (const void *pp : ptrs)
        if (!pp) return fail(GAE_ERR_INVALID_ARG, "NULL pointer in int8 attention arguments");
        else if (!aligned16(pp)) return fail(GAE_ERR_INVALID_ARG, "int8 attention pointers must be 16-byte aligned");
    if (!(a->scale >= 0.f)) return fail(GAE_ERR_UNSUPPORTED, "negative or NaN scale");
    gae::AttnParams p;
    memset(&p, 0, sizeof(p));
    gae_status s;
    // [BH, N, D] viewed as batch = BH, heads = 1.
    if ((s = make_map_4d(&p.tm_q, a->q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, BH, 1, N, D, N * D, N * D, D, 128)) != GAE_OK) return s;
    if ((s = make_map_4d(&p.tm_k, a->k, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, BH, 1, N, D, N * D, N * D, D, 128)) != GAE_OK) return s;
    if ((s = make_map_4d(&p.tm_v, a->v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, BH, 1, N, D, N * D, N * D, D, 128)) != GAE_OK) return s;
    if ((s = make_map_2d_f32(&p.tm_ks, a->k_scale, N, BH)) != GAE_OK) return s;
    p.q_scale = a->q_scale;
    p.o = a->o;
    p.lse = a->lse;
    p.o_sb = N * D; p.o_sh = N * D; p.o_ss = D;
    p.B = (int)BH; p.H = 1; p.Nq = (int)N; p.Nkv = (int)N;
    p.n_qpairs = (int)((N + 255) / 256);
    p.causal = a->causal ? 1 : 0;
    p.scale_log2 = a->scale * 1.4426950408889634f;
    const int64_t units = (int64_t)p.n_qpairs * BH;
    p.head_major = 1;
    p.logits_dump = logits_dump;
    dim3 grid((unsigned)units);  // one CTA per unit (measured faster than persistent for int8)
    if (logits_dump) return launch_tc<128, gae::kModeInt8, true>(p, grid, st);
    return launch_tc<128, gae::kModeInt8>(p, grid, st);
}

// The symphony layer's integer attention at head_dim 256 (kModeSymI8): q, k
// int8 [n, 256]; v f16 [n, 256] of which columns [half*128, half*128+128) are
// attended; o f16 [n, 256], the same columns written; ones: fp32 [n4] of 1.0
// (the per-key scale row), n4 = n rounded up to 4.  Causal.
gae_status launch_attn_sym_i8(const int8_t *q, const int8_t *k, const __half *v, __half *o, const float *ones,
                              int64_t n, int64_t n4, float scale, int half, cudaStream_t st) {
    gae::AttnParams p;
    memset(&p, 0, sizeof(p));
    gae_status s;
    if ((s = make_map_4d(&p.tm_q, q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 1, 1, n, 256, n * 256, n * 256, 256, 128)) != GAE_OK) return s;
    if ((s = make_map_4d(&p.tm_k, k, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 1, 1, n, 256, n * 256, n * 256, 256, 128)) != GAE_OK) return s;
    if ((s = make_map_4d(&p.tm_v, v + half * 128, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 1, 1, n, 128, n * 256, n * 256,
                         256, 128)) != GAE_OK)
        return s;
    if ((s = make_map_2d_f32(&p.tm_ks, ones, n4, 1)) != GAE_OK) return s;
    p.q_scale = nullptr;
    p.o = o + half * 128;
    p.o_sb = n * 256; p.o_sh = n * 256; p.o_ss = 256;
    p.B = 1; p.H = 1; p.Nq = (int)n; p.Nkv = (int)n;
    p.n_qpairs = (int)((n + 255) / 256);
    p.causal = 1;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.head_major = 1;
    return launch_tc<128, gae::kModeSymI8>(p, dim3((unsigned)p.n_qpairs), st);
}

gae_status launch_int8_logits(const int8_t *q, const int8_t *k, int64_t BH, int64_t Nq, int64_t Nkv,
                              int64_t D, int32_t *out, cudaStream_t st) {
    if (D != 128) return fail(GAE_ERR_UNSUPPORTED, "int8 logits support head_dim 128");
    if (!q || !k || !out) return fail(GAE_ERR_INVALID_ARG, "NULL pointer");
    if (!aligned16(q) || !aligned16(k)) return fail(GAE_ERR_INVALID_ARG, "q/k must be 16-byte aligned");
    if (BH > 65535) return fail(GAE_ERR_UNSUPPORTED, "batch_heads > 65535");
    gae::Int8LogitsParams p;
    memset(&p, 0, sizeof(p));
    gae_status s;
    if ((s = make_map_4d(&p.tm_q, q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, BH, 1, Nq, D, Nq * D, Nq * D, D, 128)) != GAE_OK) return s;
    if ((s = make_map_4d(&p.tm_k, k, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, BH, 1, Nkv, D, Nkv * D, Nkv * D, D, 128)) != GAE_OK) return s;
    p.out = out;
    p.Nq = (int)Nq;
    p.Nkv = (int)Nkv;
    constexpr int smem = 32768 + 64 + 1024;
    if ((s = set_smem(gae::int8_logits_kernel, smem)) != GAE_OK) return s;
    dim3 grid((unsigned)((Nq + 127) / 128), (unsigned)((Nkv + 127) / 128), (unsigned)BH);
    gae::int8_logits_kernel<<<grid, 128, smem, st>>>(p);
    GAE_CUDA_TRY(cudaGetLastError());
    return GAE_OK;
}

gae_status launch_attn_f32(const gae_attn_args *a, cudaStream_t st) {
    const int64_t D = a->head_dim;
    if (D > 256) return fail(GAE_ERR_UNSUPPORTED, "fp32 attention supports head_dim <= 256");
    gae::AttnF32Params p;
    p.q = static_cast<const float *>(a->q);
    p.k = static_cast<const float *>(a->k);
    p.v = static_cast<const float *>(a->v);
    p.o = static_cast<float *>(a->o);
    p.lse = a->lse;
    p.q_sb = a->q_stride[0]; p.q_sh = a->q_stride[1]; p.q_ss = a->q_stride[2];
    p.k_sb = a->k_stride[0]; p.k_sh = a->k_stride[1]; p.k_ss = a->k_stride[2];
    p.v_sb = a->v_stride[0]; p.v_sh = a->v_stride[1]; p.v_ss = a->v_stride[2];
    p.o_sb = a->o_stride[0]; p.o_sh = a->o_stride[1]; p.o_ss = a->o_stride[2];
    p.B = (int)a->batch; p.H = (int)a->heads; p.Nq = (int)a->seq_q; p.Nkv = (int)a->seq_kv;
    p.D = (int)D;
    p.causal = a->causal ? 1 : 0;
    p.scale = a->scale;
    p.q_offset = a->q_offset;
    p.kv_offset = a->kv_offset;
    if (a->batch * a->heads > 65535) return fail(GAE_ERR_UNSUPPORTED, "batch*heads > 65535");
    dim3 grid((unsigned)((a->seq_q + gae::kF32Rows - 1) / gae::kF32Rows),
              (unsigned)(a->batch * a->heads));
    gae_status s;
#define GAE_LAUNCH_F32(DM)                                                                   \
    do {                                                                                     \
        constexpr int smem = (DM * gae::kF32Rows + 2 * gae::kF32Keys * DM) * 4;              \
        if ((s = set_smem(gae::attn_fwd_f32_kernel<DM>, smem)) != GAE_OK) return s;         \
        gae::attn_fwd_f32_kernel<DM><<<grid, gae::kF32Rows, smem, st>>>(p);                 \
    } while (0)
    if (D <= 32) GAE_LAUNCH_F32(32);
    else if (D <= 64) GAE_LAUNCH_F32(64);
    else if (D <= 128) GAE_LAUNCH_F32(128);
    else GAE_LAUNCH_F32(256);
#undef GAE_LAUNCH_F32
    GAE_CUDA_TRY(cudaGetLastError());
    return GAE_OK;
}

gae_status check_attn_args(const gae_attn_args *a) {
    if (!a) return fail(GAE_ERR_INVALID_ARG, "args is NULL");
    if (a->batch < 1 || a->heads < 1 || a->seq_q < 0 || a->seq_kv < 0 || a->head_dim < 1)
        return fail(GAE_ERR_INVALID_ARG, "invalid shape B=%lld H=%lld Nq=%lld Nkv=%lld D=%lld",
                    (long long)a->batch, (long long)a->heads, (long long)a->seq_q,
                    (long long)a->seq_kv, (long long)a->head_dim);
    if (a->seq_q > 0 && (!a->q || !a->o))
        return fail(GAE_ERR_INVALID_ARG, "q/o pointers are NULL");
    if (a->seq_kv > 0 && (!a->k || !a->v))
        return fail(GAE_ERR_INVALID_ARG, "k/v pointers are NULL");
    if (!(a->scale == a->scale)) return fail(GAE_ERR_INVALID_ARG, "scale is NaN");
    return GAE_OK;
}

gae_status host_attention(const float *q, const float *k, const float *v, size_t n, size_t d,
                          float scale, int causal, float *out) {
    if (n == 0) return GAE_OK;
    if (!q || !k || !v || !out) return fail(GAE_ERR_INVALID_ARG, "NULL host pointer");
    if (d == 0 || d > 256) return fail(GAE_ERR_UNSUPPORTED, "head_dim must be in [1, 256]");
    const size_t bytes = n * d * sizeof(float);
    float *dq = nullptr, *dk = nullptr, *dv = nullptr, *dout = nullptr;
    gae_status s = GAE_OK;
    cudaStream_t st = nullptr;
    auto cleanup = [&] {
        if (dq) cudaFree(dq);
        if (dk) cudaFree(dk);
        if (dv) cudaFree(dv);
        if (dout) cudaFree(dout);
        if (st) cudaStreamDestroy(st);
    };
    do {
        cudaError_t e;
        if ((e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking)) != cudaSuccess ||
            (e = cudaMalloc(&dq, bytes)) != cudaSuccess || (e = cudaMalloc(&dk, bytes)) != cudaSuccess ||
            (e = cudaMalloc(&dv, bytes)) != cudaSuccess || (e = cudaMalloc(&dout, bytes)) != cudaSuccess) {
            s = fail(e == cudaErrorMemoryAllocation ? GAE_ERR_OOM : GAE_ERR_CUDA,
                     "device setup failed: %s", cudaGetErrorString(e));
            break;
        }
        if ((e = cudaMemcpyAsync(dq, q, bytes, cudaMemcpyHostToDevice, st)) != cudaSuccess ||
            (e = cudaMemcpyAsync(dk, k, bytes, cudaMemcpyHostToDevice, st)) != cudaSuccess ||
            (e = cudaMemcpyAsync(dv, v, bytes, cudaMemcpyHostToDevice, st)) != cudaSuccess) {
            s = fail(GAE_ERR_CUDA, "H2D copy failed: %s", cudaGetErrorString(e));
            break;
        }
        gae_attn_args a;
        memset(&a, 0, sizeof(a));
        a.q = dq; a.k = dk; a.v = dv; a.o = dout;
        a.batch = 1; a.heads = 1; a.seq_q = (int64_t)n; a.seq_kv = (int64_t)n; a.head_dim = (int64_t)d;
        const int64_t st3[3] = {(int64_t)(n * d), (int64_t)(n * d), (int64_t)d};
        memcpy(a.q_stride, st3, sizeof st3); memcpy(a.k_stride, st3, sizeof st3);
        memcpy(a.v_stride, st3, sizeof st3); memcpy(a.o_stride, st3, sizeof st3);
        a.dtype = GAE_DTYPE_F32;
        a.causal = causal;
        a.scale = scale;
        if ((s = launch_attn_f32(&a, st)) != GAE_OK) break;
        if ((e = cudaMemcpyAsync(out, dout, bytes, cudaMemcpyDeviceToHost, st)) != cudaSuccess ||
            (e = cudaStreamSynchronize(st)) != cudaSuccess) {
            s = fail(GAE_ERR_CUDA, "kernel or D2H copy failed: %s", cudaGetErrorString(e));
            break;
        }
    } while (0);
    cleanup();
    return s;
}

template <typename TA>
gae_status launch_merge(void *o_acc, float *lse_acc, const void *o_part, const float *lse_part,
                        int64_t rows, int64_t D, int64_t sa, int64_t sp, gae_dtype pd, cudaStream_t st) {
    const int warps = 8;
    dim3 grid((unsigned)((rows + warps - 1) / warps));
    switch (pd) {
        case GAE_DTYPE_F32:
            gae::lse_merge_kernel<TA, float><<<grid, warps * 32, 0, st>>>(
                (TA *)o_acc, lse_acc, (const float *)o_part, lse_part, rows, (int)D, sa, sp);
            break;
        case GAE_DTYPE_BF16:
            gae::lse_merge_kernel<TA, __nv_bfloat16><<<grid, warps * 32, 0, st>>>(
                (TA *)o_acc, lse_acc, (const __nv_bfloat16 *)o_part, lse_part, rows, (int)D, sa, sp);
            break;
        case GAE_DTYPE_F16:
            gae::lse_merge_kernel<TA, __half><<<grid, warps * 32, 0, st>>>(
                (TA *)o_acc, lse_acc, (const __half *)o_part, lse_part, rows, (int)D, sa, sp);
            break;
        default: return fail(GAE_ERR_INVALID_ARG, "unknown part dtype");
    }
    GAE_CUDA_TRY(cudaGetLastError());
    return GAE_OK;
}


// ------------------------------------------------------------ layer kernels
// 2-D bf16 map over a row-major [rows, cols] matrix with row stride ld
// elements, box {64, box_rows}, 128-byte swizzle (K-major GEMM operands).
gae_status make_map_kmajor(CUtensorMap *m, const void *ptr, int64_t rows, int64_t cols, int64_t ld,
                           int box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(GAE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(GAE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return GAE_OK;
}


#ifndef GAE_LINEAR_2SM
#define GAE_LINEAR_2SM 1
#endif

gae_status launch_linear(const void *x, int64_t ldx, const void *w, const float *bias, const void *res,
                         int64_t ldr, void *y, int64_t ldy, int64_t M, int64_t N, int64_t K, int epi,
                         cudaStream_t st) {
    using Cfg = gae::LinearCfg;
    if (M < 0 || N < 1 || K < 1) return fail(GAE_ERR_INVALID_ARG, "invalid linear shape");
    if (M == 0) return GAE_OK;
    if (N % Cfg::BN != 0 || K % Cfg::BK != 0)
        return fail(GAE_ERR_UNSUPPORTED, "linear needs N %% 256 == 0 and K %% 64 == 0 (N=%lld K=%lld)",
                    (long long)N, (long long)K);
    if (!x || !w || !y) return fail(GAE_ERR_INVALID_ARG, "NULL pointer");
    if (epi == gae::kEpiBiasResidual && !res) return fail(GAE_ERR_INVALID_ARG, "residual epilogue needs res");
    if (epi < 0 || epi > 2) return fail(GAE_ERR_INVALID_ARG, "unknown epilogue %d", epi);
    if (!aligned16(x) || !aligned16(w) || !aligned16(y) || (res && !aligned16(res)) || (bias && !aligned16(bias)))
        return fail(GAE_ERR_INVALID_ARG, "linear operands must be 16-byte aligned");
    if (ldx % 8 || ldy % 8 || (res && ldr % 8))
        return fail(GAE_ERR_INVALID_ARG, "row strides must be multiples of 8 elements");
    gae::LinearParams p;
    memset(&p, 0, sizeof(p));
    gae_status s;
    if ((s = make_map_kmajor(&p.tm_a, x, M, K, ldx, Cfg::BM)) != GAE_OK) return s;
    if ((s = make_map_kmajor(&p.tm_b, w, N, K, K, Cfg::BN)) != GAE_OK) return s;
    p.y = static_cast<__nv_bfloat16 *>(y);
    p.bias = bias;
    p.res = static_cast<const __nv_bfloat16 *>(res);
    p.M = (int)M; p.N = (int)N; p.K = (int)K;
    p.ldy = ldy; p.ldr = ldr;
    p.epi = epi;
    p.tiles_m = (int)((M + Cfg::BM - 1) / Cfg::BM);
    p.tiles_n = (int)(N / Cfg::BN);
#if GAE_LINEAR_2SM
    // CTA pairs on 256 x 256 tiles (the kernel derives its own tile counts).
    if ((s = make_map_kmajor(&p.tm_a, x, M, K, ldx, 128)) != GAE_OK) return s;
    if ((s = make_map_kmajor(&p.tm_b, w, N, K, K, 128)) != GAE_OK) return s;
    using Cfg2 = gae::Linear2Cfg;
    const int tiles2 = (int)((M + Cfg2::BM - 1) / Cfg2::BM) * (int)(N / Cfg2::BN);
    const int pairs = tiles2 < num_sms() / 2 ? tiles2 : num_sms() / 2;
    if ((s = set_smem(gae::linear2_kernel, Cfg2::kSmemBytes)) != GAE_OK) return s;
    gae::linear2_kernel<<<2 * pairs, Cfg2::kThreads, Cfg2::kSmemBytes, st>>>(p);
#else
    const int tiles = p.tiles_m * p.tiles_n;
    if ((s = set_smem(gae::linear_kernel, Cfg::kSmemBytes)) != GAE_OK) return s;
    const int grid = tiles < num_sms() ? tiles : num_sms();
    gae::linear_kernel<<<grid, Cfg::kThreads, Cfg::kSmemBytes, st>>>(p);
#endif
    GAE_CUDA_TRY(cudaGetLastError());
    return GAE_OK;
}

gae_status launch_layernorm(const void *x, const void *res, void *sum_out, void *y, const float *g,
                            const float *b, int64_t rows, int64_t d, float eps, cudaStream_t st) {
    if (rows == 0) return GAE_OK;
    if (!x || !y || !g || !b || rows < 0) return fail(GAE_ERR_INVALID_ARG, "invalid layernorm arguments");
    if (d % 8 != 0 || d > 8 * 32 * gae::kLnMaxChunks)
        return fail(GAE_ERR_UNSUPPORTED, "layernorm needs d %% 8 == 0 and d <= 4096");
    if (!aligned16(x) || !aligned16(y) || !aligned16(g) || !aligned16(b) || (res && !aligned16(res)) ||
        (sum_out && !aligned16(sum_out)))
        return fail(GAE_ERR_INVALID_ARG, "layernorm operands must be 16-byte aligned");
    const int warps = 8;
    // Persistent warps: two CTAs of 8 warps per SM (resident at 128
    // registers a thread), each warp walking rows.
    const int64_t blocks_needed = (rows + warps - 1) / warps;
    const int64_t blocks_cap = (int64_t)num_sms() * 2;
    dim3 grid((unsigned)(blocks_needed < blocks_cap ? blocks_needed : blocks_cap));
    const int per_lane = (int)((d + 255) / 256);
#define GAE_LN(K)                                                                                 \
    gae::layernorm_kernel<K><<<grid, warps * 32, 0, st>>>(                                        \
        (const __nv_bfloat16 *)x, (const __nv_bfloat16 *)res, (__nv_bfloat16 *)sum_out,          \
        (__nv_bfloat16 *)y, g, b, rows, (int)d, eps)
    if (per_lane <= 1) GAE_LN(1);
    else if (per_lane <= 2) GAE_LN(2);
    else if (per_lane <= 3) GAE_LN(3);
    else if (per_lane <= 4) GAE_LN(4);
    else if (per_lane <= 8) GAE_LN(8);
    else GAE_LN(16);
#undef GAE_LN
    GAE_CUDA_TRY(cudaGetLastError());
    return GAE_OK;
}

// Workspace carve-up of one layer (bytes, each region 256-byte aligned):
// ln [T, D], qkv [T, 3D], attn [T, D], x1 [T, D], hidden [T, F], and for the
// stack one spare activation [T, D].
// ok is false when a size would overflow (absurd shapes); callers reject those.
struct LayerWs {
    size_t ln, qkv, attn, x1, hid, spare, total;
    bool ok;
};
LayerWs layer_ws(int64_t T, int64_t D, int64_t F) {
    LayerWs w;
    memset(&w, 0, sizeof(w));
    const int64_t lim = (int64_t)1 << 31;
    if (T < 0 || D < 0 || F < 0 || T > lim || D > lim || F > lim) return w;
    size_t td = 0, tf = 0;
    if (__builtin_mul_overflow((size_t)T, (size_t)D * 6, &td) ||
        __builtin_mul_overflow((size_t)T, (size_t)F * 2, &tf))
        return w;
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    const size_t act = al((size_t)T * (size_t)D * 2);  // fits: T*D*6 did
    size_t o = 0;
    w.ln = o; o += act;
    w.qkv = o; o += al(td);
    w.attn = o; o += act;
    w.x1 = o; o += act;
    w.hid = o; o += al(tf);
    w.spare = o; o += act;
    w.total = o;
    w.ok = o >= td && o >= tf;  // the sum of a few in-range terms cannot wrap below them
    return w;
}

gae_status layer_once(const gae_layer_args *a, const gae_layer_weights *w, const void *x, void *out,
                      cudaStream_t st) {
    const int64_t B = a->batch, S = a->seq, D = a->d_model, Hh = a->heads, F = a->d_ff, T = B * S;
    const LayerWs L = layer_ws(T, D, F);
    char *ws = static_cast<char *>(a->workspace);
    void *ln = ws + L.ln, *qkv = ws + L.qkv, *att = ws + L.attn, *x1 = ws + L.x1, *hid = ws + L.hid;
    gae_status s;
    if ((s = launch_layernorm(x, nullptr, nullptr, ln, (const float *)w->ln1_gamma, (const float *)w->ln1_beta,
                              T, D, a->eps, st)) != GAE_OK) return s;
    if ((s = launch_linear(ln, D, w->w_qkv, (const float *)w->b_qkv, nullptr, 0, qkv, 3 * D, T, 3 * D, D,
                           gae::kEpiBias, st)) != GAE_OK) return s;
    // Causal attention straight from the packed qkv rows: head h of q/k/v is
    // columns [h*hd, (h+1)*hd) of each third; O lands in [T, D] head-major.
    const int64_t hd = D / Hh;
    gae_attn_args at;
    memset(&at, 0, sizeof(at));
    at.q = qkv;
    at.k = static_cast<char *>(qkv) + D * 2;
    at.v = static_cast<char *>(qkv) + 2 * D * 2;
    at.o = att;
    at.batch = B; at.heads = Hh; at.seq_q = S; at.seq_kv = S; at.head_dim = hd;
    const int64_t qs[3] = {S * 3 * D, hd, 3 * D}, os[3] = {S * D, hd, D};
    memcpy(at.q_stride, qs, sizeof qs); memcpy(at.k_stride, qs, sizeof qs);
    memcpy(at.v_stride, qs, sizeof qs); memcpy(at.o_stride, os, sizeof os);
    at.dtype = GAE_DTYPE_BF16;
    at.causal = 1;
    at.scale = 1.0f / sqrtf((float)hd);
    if ((s = launch_attn_tc(&at, st)) != GAE_OK) return s;
    if ((s = launch_linear(att, D, w->w_proj, (const float *)w->b_proj, x, D, x1, D, T, D, D,
                           gae::kEpiBiasResidual, st)) != GAE_OK) return s;
    if ((s = launch_layernorm(x1, nullptr, nullptr, ln, (const float *)w->ln2_gamma, (const float *)w->ln2_beta,
                              T, D, a->eps, st)) != GAE_OK) return s;
    if ((s = launch_linear(ln, D, w->w_fc, (const float *)w->b_fc, nullptr, 0, hid, F, T, F, D,
                           gae::kEpiBiasGelu, st)) != GAE_OK) return s;
    return launch_linear(hid, F, w->w_fc2, (const float *)w->b_fc2, x1, D, out, D, T, D, F,
                         gae::kEpiBiasResidual, st);
}

gae_status check_layer(const gae_layer_args *a, const gae_layer_weights *w) {
    if (!a || !w) return fail(GAE_ERR_INVALID_ARG, "args or weights NULL");
    if (a->batch < 1 || a->seq < 1 || a->d_model < 1 || a->heads < 1 || a->d_ff < 1)
        return fail(GAE_ERR_INVALID_ARG, "invalid layer shape");
    if (a->d_model % a->heads) return fail(GAE_ERR_INVALID_ARG, "d_model must be divisible by heads");
    const int64_t hd = a->d_model / a->heads;
    if (hd != 64 && hd != 128) return fail(GAE_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
    if (!a->x || !a->out || !a->workspace) return fail(GAE_ERR_INVALID_ARG, "NULL activation or workspace");
    if (a->batch > ((int64_t)1 << 31) / a->seq)
        return fail(GAE_ERR_INVALID_ARG, "batch*seq beyond 2^31 tokens");
    const LayerWs L = layer_ws(a->batch * a->seq, a->d_model, a->d_ff);
    if (!L.ok) return fail(GAE_ERR_INVALID_ARG, "layer shape too large (workspace size overflows)");
    if (a->workspace_bytes < L.total)
        return fail(GAE_ERR_INVALID_ARG, "workspace too small: %zu < %zu", a->workspace_bytes, L.total);
    const void *ps[12] = {w->ln1_gamma, w->ln1_beta, w->w_qkv, w->b_qkv, w->w_proj, w->b_proj,
                          w->ln2_gamma, w->ln2_beta, w->w_fc, w->b_fc, w->w_fc2, w->b_fc2};
    for (const void *q : ps)
        if (!q) return fail(GAE_ERR_INVALID_ARG, "NULL layer weight");
    return GAE_OK;
}
template <int D, typename TA>
gae_status launch_symphony_post(const float *x, const TA *attn, const float *w_up,
                                      const float *w_down, const float *n1, const float *n2, int64_t n,
                                      const gae::SymTuning &t, float *out, cudaStream_t st) {
    using P = gae::SymPost<D>;
    gae_status s = set_smem(gae::symphony_post_kernel<D, TA>, (int)P::kSmem);
    if (s != GAE_OK) return s;
    const unsigned blocks = (unsigned)((n + P::T - 1) / P::T);
    gae::symphony_post_kernel<D, TA><<<blocks, P::kThreads, P::kSmem, st>>>(x, attn, w_up, w_down, n1, n2, n, t, out);
    GAE_CUDA_TRY(cudaGetLastError());
    return GAE_OK;
}


// ------------------------------------------------- crate fp32 layer functions
// Device scratch of one host-memory call: every buffer is freed on scope exit.
struct HostCall {
    cudaStream_t st = nullptr;
    void *bufs[16] = {};
    int n = 0;
    ~HostCall() {
        if (st) cudaStreamSynchronize(st);
        for (int i = 0; i < n; ++i) cudaFree(bufs[i]);
        if (st) cudaStreamDestroy(st);
    }
    gae_status init() {
        GAE_CUDA_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
        return GAE_OK;
    }
    // Device copy of `count` host floats (src may be NULL: uninitialised).
    gae_status dev(float **out, const float *src, size_t count) {
        if (n >= 16) return fail(GAE_ERR_INVALID_ARG, "too many buffers");
        void *p = nullptr;
        GAE_CUDA_TRY(cudaMalloc(&p, (count ? count : 1) * sizeof(float)));
        bufs[n++] = p;
        if (src && count) GAE_CUDA_TRY(cudaMemcpyAsync(p, src, count * sizeof(float), cudaMemcpyHostToDevice, st));
        *out = static_cast<float *>(p);
        return GAE_OK;
    }
    gae_status back(float *dst, const float *src, size_t count) {
        GAE_CUDA_TRY(cudaMemcpyAsync(dst, src, count * sizeof(float), cudaMemcpyDeviceToHost, st));
        GAE_CUDA_TRY(cudaStreamSynchronize(st));
        return GAE_OK;
    }
};

gae_status launch_crate_linear(const float *x, const float *w, const float *bias, const float *res, float *y,
                               int64_t M, int64_t N, int64_t K, int w_in_major, int epi, cudaStream_t st) {
    if (M == 0 || N == 0) return GAE_OK;
    if (!x || !w || !y || M < 0 || N < 0 || K < 0) return fail(GAE_ERR_INVALID_ARG, "invalid linear arguments");
    if (epi == 2 && !res) return fail(GAE_ERR_INVALID_ARG, "residual epilogue without res");
    if (epi < 0 || epi > 2) return fail(GAE_ERR_INVALID_ARG, "unknown epilogue %d", epi);
    const int64_t gy = (M + gae::kCrateBM - 1) / gae::kCrateBM;
    if (gy > 65535) return fail(GAE_ERR_UNSUPPORTED, "more than %lld tokens", 65535LL * gae::kCrateBM);
    dim3 grid((unsigned)((N + gae::kCrateBN - 1) / gae::kCrateBN), (unsigned)gy);
    if (w_in_major)
        gae::crate_linear_f32_kernel<true><<<grid, 256, 0, st>>>(x, w, bias, res, y, M, N, K, epi);
    else
        gae::crate_linear_f32_kernel<false><<<grid, 256, 0, st>>>(x, w, bias, res, y, M, N, K, epi);
    GAE_CUDA_TRY(cudaGetLastError());
    return GAE_OK;
}

gae_status launch_crate_layernorm(const float *x, const float *g, const float *b, float *y, int64_t rows,
                                  int64_t d, float eps, cudaStream_t st) {
    if (rows == 0 || d == 0) return GAE_OK;
    if (!x || !g || !b || !y || rows < 0 || d < 0) return fail(GAE_ERR_INVALID_ARG, "invalid layernorm arguments");
    const int64_t blocks = (rows + 127) / 128;
    if (blocks > INT32_MAX) return fail(GAE_ERR_UNSUPPORTED, "too many rows");
    gae::crate_layernorm_f32_kernel<<<(unsigned)blocks, 128, 0, st>>>(x, g, b, y, rows, d, eps);
    GAE_CUDA_TRY(cudaGetLastError());
    return GAE_OK;
}

// LayerNorm(mlp_block(x) + residual) over `tokens` rows (mlp.rs:39-73); on
// device buffers, hid [tokens, mlp] and tmp [tokens, hidden] scratch.
gae_status crate_fused_mlp_ln(const float *x, const float *res, const float *w1, const float *b1,
                              const float *w2, const float *b2, const float *g, const float *bt,
                              int64_t T, int64_t h, int64_t m, float eps, float *hid, float *tmp,
                              float *out, cudaStream_t st) {
    gae_status s;
    if ((s = launch_crate_linear(x, w1, b1, nullptr, hid, T, m, h, 1, 1, st)) != GAE_OK) return s;
    if ((s = launch_crate_linear(hid, w2, b2, res, tmp, T, h, m, 1, 2, st)) != GAE_OK) return s;
    return launch_crate_layernorm(tmp, g, bt, out, T, h, eps, st);
}

bool mul_ok(size_t a, size_t b, size_t *out) { return !__builtin_mul_overflow(a, b, out); }
}  // namespace

#include "ring.cuh"

// ==================================================================== C ABI
extern "C" {

const char *gae_status_string(gae_status s) {
    switch (s) {
        case GAE_OK: return "GAE_OK";
        case GAE_ERR_INVALID_ARG: return "GAE_ERR_INVALID_ARG";
        case GAE_ERR_UNSUPPORTED: return "GAE_ERR_UNSUPPORTED";
        case GAE_ERR_CUDA: return "GAE_ERR_CUDA";
        case GAE_ERR_OOM: return "GAE_ERR_OOM";
        case GAE_ERR_COMM: return "GAE_ERR_COMM";
        case GAE_ERR_TIMEOUT: return "GAE_ERR_TIMEOUT";
    }
    return "GAE_ERR_UNKNOWN";
}

gae_status gae_last_error(char *buf, size_t n) {
    if (buf && n) {
        strncpy(buf, g_err, n - 1);
        buf[n - 1] = '\0';
    }
    return g_err_status;
}

const char *gae_version(void) { return "0.1.0"; }

gae_status gae_device_status(int reset) {
    GAE_CUDA_TRY(cudaDeviceSynchronize());
    unsigned v = 0;
    GAE_CUDA_TRY(cudaMemcpyFromSymbol(&v, gae::gae_dev_error, sizeof(v)));
    if (reset) {
        unsigned z = 0;
        GAE_CUDA_TRY(cudaMemcpyToSymbol(gae::gae_dev_error, &z, sizeof(z)));
    }
    if (v) return fail(GAE_ERR_TIMEOUT, "a device-side wait timed out (site 0x%x)", v);
    return GAE_OK;
}

namespace gae {
// One thread waits, with a bounded wait, on an mbarrier that nothing arrives
// on: the wait gives up after timeout_ns, records `site` and returns; no
// asynchronous copy or MMA is in flight, so the kernel exits cleanly.
__global__ void wait_timeout_probe_kernel(uint64_t timeout_ns, unsigned site) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait_for(smem_u32(&bar), 0, site, &abort_flag, timeout_ns);
}
}  // namespace gae

extern "C" gae_status gae_debug_attn_int8_logits(const gae_attn_int8_args *a, int32_t *logits, void *stream) {
    if (!a || !logits) return fail(GAE_ERR_INVALID_ARG, "args or logits NULL");
    if (a->batch_heads < 1 || a->seq < 0 || a->head_dim < 1)
        return fail(GAE_ERR_INVALID_ARG, "invalid int8 attention shape");
    if (a->seq == 0) return GAE_OK;
    return launch_attn_int8(a, static_cast<cudaStream_t>(stream), logits);
}

extern "C" gae_status gae_debug_wait_timeout(uint64_t timeout_ns, void *stream) {
    if (timeout_ns > 1000000000ull) return fail(GAE_ERR_INVALID_ARG, "timeout above 1 s");
    gae::wait_timeout_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(timeout_ns, 0x901u);
    GAE_CUDA_TRY(cudaGetLastError());
    return GAE_OK;
}

gae_status gae_debug_attn_trace(void *buf, int cta) {
#ifndef GAE_ATTN_TRACE
    (void)buf; (void)cta;
    return fail(GAE_ERR_UNSUPPORTED, "this build has no attention trace (compile with -DGAE_ATTN_TRACE)");
#endif
    unsigned long long *p = static_cast<unsigned long long *>(buf);
    GAE_CUDA_TRY(cudaMemcpyToSymbol(gae::gae_attn_trace, &p, sizeof(p)));
    GAE_CUDA_TRY(cudaMemcpyToSymbol(gae::gae_attn_trace_cta, &cta, sizeof(cta)));
    return GAE_OK;
}

gae_status gae_waller_operator_f32_host(const float *q, const float *k, const float *v,
                                        size_t seq_len, size_t head_dim, float scale, int causal,
                                        float *out) {
    return host_attention(q, k, v, seq_len, head_dim, scale, causal, out);
}

gae_status gae_waller_operator_parallel_f32_host(const float *q, const float *k, const float *v,
                                                 size_t seq_len, size_t head_dim, float scale,
                                                 int causal, float *out) {
    return host_attention(q, k, v, seq_len, head_dim, scale, causal, out);
}

gae_status gae_standard_attention_f32_host(const float *q, const float *k, const float *v,
                                           size_t seq_len, size_t head_dim, float scale,
                                           int causal, float *out) {
    return host_attention(q, k, v, seq_len, head_dim, scale, causal, out);
}

gae_status gae_attn_fwd(const gae_attn_args *a, void *stream) {
    gae_status s = check_attn_args(a);
    if (s != GAE_OK) return s;
    if (a->seq_q == 0) return GAE_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (a->dtype) {
        case GAE_DTYPE_F32: return launch_attn_f32(a, st);
        case GAE_DTYPE_BF16:
        case GAE_DTYPE_F16: return launch_attn_tc(a, st);
    }
    return fail(GAE_ERR_INVALID_ARG, "unknown dtype %d", (int)a->dtype);
}

gae_status gae_lse_merge(void *o_acc, float *lse_acc, const void *o_part, const float *lse_part,
                         int64_t rows, int64_t head_dim, int64_t sa, int64_t sp, gae_dtype ad,
                         gae_dtype pd, void *stream) {
    if (rows == 0) return GAE_OK;
    if (!o_acc || !lse_acc || !o_part || !lse_part || rows < 0 || head_dim < 1 || sa < head_dim ||
        sp < head_dim)
        return fail(GAE_ERR_INVALID_ARG, "invalid lse_merge arguments");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (ad) {
        case GAE_DTYPE_F32: return launch_merge<float>(o_acc, lse_acc, o_part, lse_part, rows, head_dim, sa, sp, pd, st);
        case GAE_DTYPE_BF16: return launch_merge<__nv_bfloat16>(o_acc, lse_acc, o_part, lse_part, rows, head_dim, sa, sp, pd, st);
        case GAE_DTYPE_F16: return launch_merge<__half>(o_acc, lse_acc, o_part, lse_part, rows, head_dim, sa, sp, pd, st);
    }
    return fail(GAE_ERR_INVALID_ARG, "unknown acc dtype");
}

size_t gae_layer_workspace_bytes(int64_t batch, int64_t seq, int64_t d_model, int64_t d_ff) {
    if (batch < 1 || seq < 1 || d_model < 1 || d_ff < 1) return 0;
    if (batch > ((int64_t)1 << 31) / seq) return 0;
    const LayerWs L = layer_ws(batch * seq, d_model, d_ff);
    return L.ok ? L.total : 0;
}

gae_status gae_layer_fwd(const gae_layer_args *a, const gae_layer_weights *w, void *stream) {
    gae_status s = check_layer(a, w);
    if (s != GAE_OK) return s;
    return layer_once(a, w, a->x, a->out, static_cast<cudaStream_t>(stream));
}

gae_status gae_layer_stack_fwd(const gae_layer_args *a, const gae_layer_weights *w, int n_layers,
                               void *stream) {
    gae_status s = check_layer(a, w);
    if (s != GAE_OK) return s;
    if (n_layers < 1) return fail(GAE_ERR_INVALID_ARG, "n_layers must be >= 1");
    for (int i = 0; i < n_layers; ++i)
        if ((s = check_layer(a, w + i)) != GAE_OK) return s;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const LayerWs L = layer_ws(a->batch * a->seq, a->d_model, a->d_ff);
    void *spare = static_cast<char *>(a->workspace) + L.spare;
    // Layer i reads cur and writes out when n_layers-1-i is even, else the
    // spare buffer, so the last layer lands in out.  A layer may run in place
    // (its input is last read by the projection, before its output is written).
    const void *cur = a->x;
    for (int i = 0; i < n_layers; ++i) {
        void *nxt = ((n_layers - 1 - i) % 2 == 0) ? a->out : spare;
        if ((s = layer_once(a, w + i, cur, nxt, st)) != GAE_OK) return s;
        cur = nxt;
    }
    return GAE_OK;
}

size_t gae_attn_bwd_workspace_bytes(int64_t batch, int64_t heads, int64_t seq_q, int64_t head_dim) {
    if (batch < 1 || heads < 1 || seq_q < 1 || head_dim < 1) return 0;
    return attn_bwd_ws_region(batch, heads, seq_q, head_dim) +
           (((size_t)(batch * heads * seq_q) * 4 + 255) & ~(size_t)255);
}

gae_status gae_attn_bwd(const gae_attn_bwd_args *args, void *stream) {
    if (!args) return fail(GAE_ERR_INVALID_ARG, "NULL args");
    return launch_attn_bwd(args, static_cast<cudaStream_t>(stream));
}

size_t gae_symphony_workspace_bytes(int64_t seq_len, int64_t head_dim) {
    if (seq_len < 1 || head_dim < 1) return 0;
    const size_t region = ((size_t)seq_len * head_dim * 2 + 255) & ~(size_t)255;
    if (head_dim == 256)  // q int8, v f16, the attention output f16, a row of ones
        return 3 * region + ((((size_t)seq_len + 3) / 4 * 16 + 255) & ~(size_t)255);
    return 4 * region;  // q, k, v (f16) and the attention output (f16)
}

gae_status gae_symphony_fwd(const float *input, const int8_t *k, const int8_t *v, const float *w_up,
                            const float *w_down, const float *norm1_w, const float *norm2_w,
                            int64_t n, int64_t d, const gae_tuning_fork *tf, float *output,
                            void *workspace, size_t workspace_bytes, void *stream) {
    if (n == 0) return GAE_OK;
    if (!input || !k || !v || !w_up || !w_down || !norm1_w || !norm2_w || !tf || !output || !workspace)
        return fail(GAE_ERR_INVALID_ARG, "NULL pointer in symphony arguments");
    if (n < 0 || (d != 64 && d != 128 && d != 256))
        return fail(GAE_ERR_UNSUPPORTED, "symphony supports head_dim 64, 128 or 256");
    if (!(tf->attn_temperature != 0.f)) return fail(GAE_ERR_INVALID_ARG, "attn_temperature is zero");
    const size_t need = gae_symphony_workspace_bytes(n, d);
    if (workspace_bytes < need) return fail(GAE_ERR_INVALID_ARG, "workspace too small: %zu < %zu", workspace_bytes, need);
    if (!aligned16(workspace) || !aligned16(input) || !aligned16(output) || !aligned16(w_up) || !aligned16(w_down))
        return fail(GAE_ERR_INVALID_ARG, "symphony: input, output, weights and workspace must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t region = need / 4;
    char *ws = static_cast<char *>(workspace);
    const int64_t elems = n * d;
    gae_attn_args a;
    memset(&a, 0, sizeof(a));
    a.q = ws; a.k = ws + region; a.v = ws + 2 * region; a.o = ws + 3 * region;
    a.batch = 1; a.heads = 1; a.seq_q = n; a.seq_kv = n; a.head_dim = d;
    const int64_t str[3] = {n * d, n * d, d};
    memcpy(a.q_stride, str, sizeof str); memcpy(a.k_stride, str, sizeof str);
    memcpy(a.v_stride, str, sizeof str); memcpy(a.o_stride, str, sizeof str);
    a.causal = 1;
    a.scale = tf->attn_scale / tf->attn_temperature;
    if (!(a.scale >= 0.f)) return fail(GAE_ERR_UNSUPPORTED, "attn_scale / attn_temperature must be >= 0");
    gae_status s;
    if (d == 256) {
        // head_dim 256: QK^T over the 256 int8 dimensions on the int8 tensor
        // cores (exact int32 dots, the reference's own arithmetic), P*V in
        // two launches over the two 128-column halves of V (TMEM holds two
        // 128-row Q tiles' S and O up to 128 columns of O each); S is
        // recomputed by the second launch at the int8 rate.
        const size_t region = ((size_t)n * d * 2 + 255) & ~(size_t)255;
        int8_t *q8 = reinterpret_cast<int8_t *>(ws);
        __half *vh = reinterpret_cast<__half *>(ws + region);
        __half *oh16 = reinterpret_cast<__half *>(ws + 2 * region);
        float *ones = reinterpret_cast<float *>(ws + 3 * region);
        const int64_t n4 = (n + 3) / 4 * 4;
        gae::symphony_prep_i8_kernel<<<(unsigned)((elems + 255) / 256), 256, 0, st>>>(input, v, q8, vh, ones, elems,
                                                                                      n4);
        GAE_CUDA_TRY(cudaGetLastError());
        if (!aligned16(k)) return fail(GAE_ERR_INVALID_ARG, "symphony: k must be 16-byte aligned at head_dim 256");
        for (int half = 0; half < 2; ++half)
            if ((s = launch_attn_sym_i8(q8, k, vh, oh16, ones, n, n4, a.scale, half, st)) != GAE_OK) return s;
        a.o = oh16;
    } else {
        gae::symphony_prep_kernel<__half><<<(unsigned)((elems + 255) / 256), 256, 0, st>>>(
            input, k, v, (__half *)a.q, (__half *)a.k, (__half *)a.v, elems);
        GAE_CUDA_TRY(cudaGetLastError());
        a.dtype = GAE_DTYPE_F16;
        if ((s = launch_attn_tc(&a, st)) != GAE_OK) return s;
    }
    gae::SymTuning t;
    t.attn_scale = tf->attn_scale; t.attn_temperature = tf->attn_temperature;
    t.residual_alpha = tf->residual_alpha; t.residual_beta = tf->residual_beta; t.norm_eps = tf->norm_eps;
    t.activation_type = tf->activation_type; t.mlp_gate = tf->mlp_gate; t.output_scale = tf->output_scale;
    const __half *oh = static_cast<const __half *>(a.o);
    if (d == 64) s = launch_symphony_post<64>(input, oh, w_up, w_down, norm1_w, norm2_w, n, t, output, st);
    else if (d == 128) s = launch_symphony_post<128>(input, oh, w_up, w_down, norm1_w, norm2_w, n, t, output, st);
    else s = launch_symphony_post<256>(input, oh, w_up, w_down, norm1_w, norm2_w, n, t, output, st);
    if (s != GAE_OK) return s;
    GAE_CUDA_TRY(cudaGetLastError());
    return GAE_OK;
}

gae_status gae_layernorm_fwd(const void *x, const void *res, void *sum_out, void *y, const float *gamma,
                             const float *beta, int64_t rows, int64_t d, float eps, void *stream) {
    return launch_layernorm(x, res, sum_out, y, gamma, beta, rows, d, eps, static_cast<cudaStream_t>(stream));
}

gae_status gae_linear_fwd(const void *x, const void *w, const float *bias, const void *res, void *y,
                          int64_t M, int64_t N, int64_t K, int epilogue, void *stream) {
    return launch_linear(x, K, w, bias, res, N, y, N, M, N, K, epilogue, static_cast<cudaStream_t>(stream));
}

gae_status gae_attn_int8_fwd(const gae_attn_int8_args *a, void *stream) {
    if (!a) return fail(GAE_ERR_INVALID_ARG, "args is NULL");
    if (a->batch_heads < 1 || a->seq < 0 || a->head_dim < 1)
        return fail(GAE_ERR_INVALID_ARG, "invalid int8 attention shape");
    if (a->seq == 0) return GAE_OK;
    return launch_attn_int8(a, static_cast<cudaStream_t>(stream));
}

gae_status gae_int8_logits(const int8_t *q, const int8_t *k, int64_t batch_heads, int64_t seq_q,
                           int64_t seq_kv, int64_t head_dim, int32_t *logits, void *stream) {
    if (batch_heads < 1 || seq_q < 0 || seq_kv < 0 || head_dim < 1)
        return fail(GAE_ERR_INVALID_ARG, "invalid int8 logits shape");
    if (seq_q == 0 || seq_kv == 0) return GAE_OK;
    return launch_int8_logits(q, k, batch_heads, seq_q, seq_kv, head_dim, logits,
                              static_cast<cudaStream_t>(stream));
}

gae_status gae_quantize_rows_int8(const void *x, gae_dtype dtype, int64_t rows, int64_t d,
                                  int8_t *q, float *scale, void *stream) {
    if (rows == 0) return GAE_OK;
    if (!x || !q || !scale || rows < 0 || d < 1)
        return fail(GAE_ERR_INVALID_ARG, "invalid quantize arguments");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int warps = 8;
    dim3 grid((unsigned)((rows + warps - 1) / warps));
    if (dtype == GAE_DTYPE_F32)
        gae::quantize_rows_int8_kernel<float><<<grid, warps * 32, 0, st>>>((const float *)x, rows, (int)d, q, scale);
    else if (dtype == GAE_DTYPE_BF16)
        gae::quantize_rows_int8_kernel<__nv_bfloat16><<<grid, warps * 32, 0, st>>>(
            (const __nv_bfloat16 *)x, rows, (int)d, q, scale);
    else
        return fail(GAE_ERR_UNSUPPORTED, "quantize supports f32 and bf16 input");
    GAE_CUDA_TRY(cudaGetLastError());
    return GAE_OK;
}


// ------------------------------------------------- crate fp32 layer functions
gae_status gae_crate_linear_f32(const float *x, const float *w, const float *bias, const float *res, float *y,
                                int64_t M, int64_t N, int64_t K, int w_in_major, int epilogue, void *stream) {
    return launch_crate_linear(x, w, bias, res, y, M, N, K, w_in_major, epilogue,
                               static_cast<cudaStream_t>(stream));
}

gae_status gae_crate_layernorm_f32(const float *x, const float *gamma, const float *beta, float *y,
                                   int64_t rows, int64_t d, float eps, void *stream) {
    return launch_crate_layernorm(x, gamma, beta, y, rows, d, eps, static_cast<cudaStream_t>(stream));
}

gae_status gae_layernorm_batched_f32_host(const float *input, const float *gamma, const float *beta,
                                          size_t batch, size_t hidden, float eps, float *out) {
    size_t n = 0;
    if (!mul_ok(batch, hidden, &n)) return fail(GAE_ERR_INVALID_ARG, "batch*hidden overflows");
    if (n == 0) return GAE_OK;
    if (!input || !gamma || !beta || !out) return fail(GAE_ERR_INVALID_ARG, "NULL host pointer");
    HostCall c;
    float *dx, *dg, *db, *dy;
    gae_status s;
    if ((s = c.init()) || (s = c.dev(&dx, input, n)) || (s = c.dev(&dg, gamma, hidden)) ||
        (s = c.dev(&db, beta, hidden)) || (s = c.dev(&dy, nullptr, n)))
        return s;
    if ((s = launch_crate_layernorm(dx, dg, db, dy, (int64_t)batch, (int64_t)hidden, eps, c.st))) return s;
    return c.back(out, dy, n);
}

gae_status gae_layernorm_f32_host(const float *input, const float *gamma, const float *beta, size_t n,
                                  float eps, float *out) {
    return gae_layernorm_batched_f32_host(input, gamma, beta, n ? 1 : 0, n, eps, out);
}

gae_status gae_mlp_block_f32_host(const float *input, const float *w1, const float *b1, const float *w2,
                                  const float *b2, size_t hidden_dim, size_t mlp_dim, size_t tokens,
                                  float *out) {
    size_t nx = 0, nh = 0, nw = 0;
    if (!mul_ok(tokens, hidden_dim, &nx) || !mul_ok(tokens, mlp_dim, &nh) || !mul_ok(hidden_dim, mlp_dim, &nw))
        return fail(GAE_ERR_INVALID_ARG, "size overflows");
    if (nx == 0) return GAE_OK;
    if (!input || !w1 || !b1 || !w2 || !b2 || !out) return fail(GAE_ERR_INVALID_ARG, "NULL host pointer");
    HostCall c;
    float *dx, *dw1, *db1, *dw2, *db2, *dh, *dy;
    gae_status s;
    if ((s = c.init()) || (s = c.dev(&dx, input, nx)) || (s = c.dev(&dw1, w1, nw)) ||
        (s = c.dev(&db1, b1, mlp_dim)) || (s = c.dev(&dw2, w2, nw)) || (s = c.dev(&db2, b2, hidden_dim)) ||
        (s = c.dev(&dh, nullptr, nh)) || (s = c.dev(&dy, nullptr, nx)))
        return s;
    const int64_t T = (int64_t)tokens, h = (int64_t)hidden_dim, m = (int64_t)mlp_dim;
    if ((s = launch_crate_linear(dx, dw1, db1, nullptr, dh, T, m, h, 1, 1, c.st))) return s;
    if ((s = launch_crate_linear(dh, dw2, db2, nullptr, dy, T, h, m, 1, 0, c.st))) return s;
    return c.back(out, dy, nx);
}

gae_status gae_fused_mlp_layernorm_f32_host(const float *input, const float *residual, const float *w1,
                                            const float *b1, const float *w2, const float *b2,
                                            const float *gamma, const float *beta, size_t hidden_dim,
                                            size_t mlp_dim, float eps, size_t tokens, float *out) {
    size_t nx = 0, nh = 0, nw = 0;
    if (!mul_ok(tokens, hidden_dim, &nx) || !mul_ok(tokens, mlp_dim, &nh) || !mul_ok(hidden_dim, mlp_dim, &nw))
        return fail(GAE_ERR_INVALID_ARG, "size overflows");
    if (nx == 0) return GAE_OK;
    if (!input || !residual || !w1 || !b1 || !w2 || !b2 || !gamma || !beta || !out)
        return fail(GAE_ERR_INVALID_ARG, "NULL host pointer");
    HostCall c;
    float *dx, *dr, *dw1, *db1, *dw2, *db2, *dg, *dbt, *dh, *dt, *dy;
    gae_status s;
    if ((s = c.init()) || (s = c.dev(&dx, input, nx)) || (s = c.dev(&dr, residual, nx)) ||
        (s = c.dev(&dw1, w1, nw)) || (s = c.dev(&db1, b1, mlp_dim)) || (s = c.dev(&dw2, w2, nw)) ||
        (s = c.dev(&db2, b2, hidden_dim)) || (s = c.dev(&dg, gamma, hidden_dim)) ||
        (s = c.dev(&dbt, beta, hidden_dim)) || (s = c.dev(&dh, nullptr, nh)) || (s = c.dev(&dt, nullptr, nx)) ||
        (s = c.dev(&dy, nullptr, nx)))
        return s;
    if ((s = crate_fused_mlp_ln(dx, dr, dw1, db1, dw2, db2, dg, dbt, (int64_t)tokens, (int64_t)hidden_dim,
                                (int64_t)mlp_dim, eps, dh, dt, dy, c.st)))
        return s;
    return c.back(out, dy, nx);
}

gae_status gae_transformer_block_forward_f32_host(const gae_transformer_block_f32 *b, const float *input,
                                                  size_t seq_len, float *out) {
    if (!b) return fail(GAE_ERR_INVALID_ARG, "block is NULL");
    const size_t h = b->hidden_dim, m = b->mlp_dim;
    size_t nx = 0, nh = 0, nw = 0, nhh = 0;
    if (!mul_ok(seq_len, h, &nx) || !mul_ok(seq_len, m, &nh) || !mul_ok(h, m, &nw) || !mul_ok(h, h, &nhh))
        return fail(GAE_ERR_INVALID_ARG, "size overflows");
    if (nx == 0) return GAE_OK;
    if (h == 0 || m == 0) return fail(GAE_ERR_INVALID_ARG, "hidden_dim and mlp_dim must be positive");
    if (!input || !out || !b->wv || !b->wo || !b->ln1_gamma || !b->ln1_beta || !b->w1 || !b->b1 || !b->w2 ||
        !b->b2 || !b->ln2_gamma || !b->ln2_beta)
        return fail(GAE_ERR_INVALID_ARG, "NULL host pointer");
    HostCall c;
    float *dx, *dwv, *dwo, *dg1, *db1n, *dw1, *db1, *dw2, *db2, *dg2, *db2n, *dn, *dv, *dr1, *dh, *dt;
    gae_status s;
    if ((s = c.init()) || (s = c.dev(&dx, input, nx)) || (s = c.dev(&dwv, b->wv, nhh)) ||
        (s = c.dev(&dwo, b->wo, nhh)) || (s = c.dev(&dg1, b->ln1_gamma, h)) || (s = c.dev(&db1n, b->ln1_beta, h)) ||
        (s = c.dev(&dw1, b->w1, nw)) || (s = c.dev(&db1, b->b1, m)) || (s = c.dev(&dw2, b->w2, nw)) ||
        (s = c.dev(&db2, b->b2, h)) || (s = c.dev(&dg2, b->ln2_gamma, h)) || (s = c.dev(&db2n, b->ln2_beta, h)) ||
        (s = c.dev(&dn, nullptr, nx)) || (s = c.dev(&dv, nullptr, nx)) || (s = c.dev(&dr1, nullptr, nx)) ||
        (s = c.dev(&dh, nullptr, nh)) || (s = c.dev(&dt, nullptr, nx)))
        return s;
    const int64_t T = (int64_t)seq_len, H = (int64_t)h, M = (int64_t)m;
    // transformer.rs:97-116, every token independently: LN1 -> Wv -> Wo + x ->
    // LN2(MLP(r1) + r1).  dn is reused for the final output.
    if ((s = launch_crate_layernorm(dx, dg1, db1n, dn, T, H, b->eps, c.st))) return s;
    if ((s = launch_crate_linear(dn, dwv, nullptr, nullptr, dv, T, H, H, 0, 0, c.st))) return s;
    if ((s = launch_crate_linear(dv, dwo, nullptr, dx, dr1, T, H, H, 0, 2, c.st))) return s;
    if ((s = crate_fused_mlp_ln(dr1, dr1, dw1, db1, dw2, db2, dg2, db2n, T, H, M, b->eps, dh, dt, dn, c.st)))
        return s;
    return c.back(out, dn, nx);
}

// ------------------------------------------------- sequence-parallel ring
gae_status gae_ring_unique_id(void *unique_id) {
    if (!unique_id) return fail(GAE_ERR_INVALID_ARG, "unique_id is NULL");
    const NcclApi *nc = nccl_api();
    if (!nc) return fail(GAE_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
    ncclUniqueId id;
    const ncclResult_t r = nc->GetUniqueId(&id);
    if (r != ncclSuccess) return fail(GAE_ERR_COMM, "ncclGetUniqueId: %s", nc->GetErrorString(r));
    static_assert(sizeof(ncclUniqueId) == GAE_RING_UNIQUE_ID_BYTES, "unique id size");
    memcpy(unique_id, &id, sizeof(id));
    return GAE_OK;
}

gae_status gae_ring_ctx_create(const void *unique_id, int rank, int world, double timeout_s, gae_ring_ctx **out) {
    if (!out || (!unique_id && world > 1)) return fail(GAE_ERR_INVALID_ARG, "NULL argument");
    *out = nullptr;
    if (world < 1 || rank < 0 || rank >= world) return fail(GAE_ERR_INVALID_ARG, "rank %d of world %d", rank, world);
    if (world == 1) {  // the whole sequence is local: no communicator (and no NCCL) needed
        gae_ring_ctx *c = new gae_ring_ctx();
        c->world = 1;
        c->timeout_s = timeout_s;
        gae_status s = ring_ctx_init_common(c);
        if (s != GAE_OK) {
            ring_ctx_release(c);
            return s;
        }
        *out = c;
        return GAE_OK;
    }
    const NcclApi *nc = nccl_api();
    if (!nc) return fail(GAE_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
    gae_ring_ctx *c = new gae_ring_ctx();
    c->nc = nc;
    c->rank = rank;
    c->world = world;
    c->timeout_s = timeout_s;
    gae_status s = ring_ctx_init_common(c);
    if (s == GAE_OK) {
        ncclUniqueId id;
        memcpy(&id, unique_id, sizeof(id));
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;  // every wait is bounded by the timeout
        const ncclResult_t r = nc->CommInitRankConfig(&c->comm, world, id, rank, &cfg);
        c->owns_comm = true;
        if (r != ncclSuccess && r != ncclInProgress)
            s = fail(GAE_ERR_COMM, "ncclCommInitRankConfig: %s", nc->GetErrorString(r));
        else
            s = nccl_settle(c, r, "joining the communicator");
    }
    if (s != GAE_OK) {
        const gae_status keep = g_err_status;
        char msg[sizeof g_err];
        memcpy(msg, g_err, sizeof msg);
        ring_ctx_release(c);
        g_err_status = keep;
        memcpy(g_err, msg, sizeof msg);
        return s;
    }
    *out = c;
    return GAE_OK;
}

gae_status gae_ring_ctx_create_from_comm(void *nccl_comm, double timeout_s, gae_ring_ctx **out) {
    if (!out || !nccl_comm) return fail(GAE_ERR_INVALID_ARG, "NULL argument");
    *out = nullptr;
    const NcclApi *nc = nccl_api();
    if (!nc) return fail(GAE_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
    gae_ring_ctx *c = new gae_ring_ctx();
    c->nc = nc;
    c->comm = static_cast<ncclComm_t>(nccl_comm);
    c->owns_comm = false;
    c->timeout_s = timeout_s;
    gae_status s = ring_ctx_init_common(c);
    if (s == GAE_OK && (nc->CommCount(c->comm, &c->world) != ncclSuccess ||
                        nc->CommUserRank(c->comm, &c->rank) != ncclSuccess))
        s = fail(GAE_ERR_COMM, "the communicator reports no rank/size");
    if (s != GAE_OK) {
        ring_ctx_release(c);
        return s;
    }
    *out = c;
    return GAE_OK;
}

gae_status gae_ring_ctx_destroy(gae_ring_ctx *ctx) {
    if (ctx) ring_ctx_release(ctx);
    return GAE_OK;
}

gae_status gae_ring_attn_fwd(gae_ring_ctx *ctx, const gae_attn_args *a, int balance, void *stream) {
    int zig = 0;
    gae_status s = ring_check_args(ctx, a, balance, &zig);
    if (s != GAE_OK) return s;
    if (a->seq_q == 0) return GAE_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int dev = -1;
    GAE_CUDA_TRY(cudaGetDevice(&dev));
    if (dev != ctx->device) return fail(GAE_ERR_INVALID_ARG, "current device %d is not the context's %d", dev, ctx->device);
    if (ctx->world == 1) return launch_attn_tc(a, st);  // the whole sequence is here: one launch
    if (ctx->comm) {
        ncclResult_t as = ncclSuccess;
        if (ctx->nc->CommGetAsyncError(ctx->comm, &as) != ncclSuccess || (as != ncclSuccess && as != ncclInProgress))
            return ring_fail(ctx, GAE_ERR_COMM, "communicator", ctx->nc->GetErrorString(as));
    }
    s = a->dtype == GAE_DTYPE_BF16 ? ring_run<__nv_bfloat16>(ctx, a, zig, st) : ring_run<__half>(ctx, a, zig, st);
    if (s != GAE_OK) return s;
    if (ctx->timeout_s > 0) {
        GAE_CUDA_TRY(cudaEventRecord(ctx->ev_done, st));
        return ring_wait_event(ctx, ctx->ev_done, "waiting for the ring to finish");
    }
    return GAE_OK;
}

gae_status gae_debug_ring_plan(int rank, int world, int step, int causal, int zigzag, int64_t shard_len,
                               int64_t *ops, int *n_ops) {
    if (!ops || !n_ops || world < 1 || rank < 0 || rank >= world || step < 0 || step >= world || shard_len < 0)
        return fail(GAE_ERR_INVALID_ARG, "invalid ring plan query");
    RingOp o[2];
    const int n = ring_plan(rank, world, step, causal, zigzag, shard_len, o);
    for (int i = 0; i < n; ++i) {
        const int64_t v[7] = {o[i].q_row0, o[i].q_rows, o[i].kv_row0, o[i].kv_rows, o[i].causal, o[i].q_pos,
                              o[i].kv_pos};
        memcpy(ops + 7 * i, v, sizeof v);
    }
    *n_ops = n;
    return GAE_OK;
}
}  // extern "C"

// ====================================================================
// Allocation-free layer forward.
//
// Some callers cannot allocate device memory for the layer's workspace: code
// running inside an allocator or memory-pool callback, plugins whose host
// application owns every device allocation and forbids cudaMalloc, or
// real-time paths where an allocation may block.  gae_layer_fwd_static runs
// the same kernels as gae_layer_fwd but takes its workspace from a
// file-scope device array of kStaticLayerWsBytes, which every GPU that loads
// this library holds until the process exits.  It calls no cudaMalloc,
// cudaFree or other allocating routine.
namespace {

constexpr size_t kStaticLayerWsBytes = 32ull << 20;  // 32 MiB per device
static __device__ __align__(256) unsigned char g_layer_static_ws[kStaticLayerWsBytes];

constexpr int kStaticMaxDevices = 64;
std::mutex g_static_ws_mu;
void *g_static_ws_ptr[kStaticMaxDevices] = {};
CUcontext g_static_ws_ctx[kStaticMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext *);
CtxGetCurrentFn ctx_get_current_fn() {
    static CtxGetCurrentFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<CtxGetCurrentFn>(p);
    }();
    return fn;
}

// Device address of the array on the current device.  Host code may not use
// the array's name as a pointer (it is only a host-side stand-in), so the
// address is looked up once per device, with that device current.  The
// context it was looked up in is kept beside it: after a cudaDeviceReset (a
// new primary context, the module loaded again, perhaps elsewhere) the
// address is looked up afresh instead of reusing a stale one.
gae_status static_ws_address(void **out) {
    int dev = 0;
    GAE_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kStaticMaxDevices)
        return fail(GAE_ERR_UNSUPPORTED, "device index %d beyond %d", dev, kStaticMaxDevices);
    CtxGetCurrentFn get_ctx = ctx_get_current_fn();
    if (!get_ctx) return fail(GAE_ERR_CUDA, "cuCtxGetCurrent is unavailable");
    CUcontext ctx = nullptr;
    get_ctx(&ctx);
    std::lock_guard<std::mutex> lock(g_static_ws_mu);
    if (!ctx || !g_static_ws_ptr[dev] || g_static_ws_ctx[dev] != ctx) {
        void *p = nullptr;
        GAE_CUDA_TRY(cudaGetSymbolAddress(&p, g_layer_static_ws));  // also makes the context current
        if (!p) return fail(GAE_ERR_CUDA, "cudaGetSymbolAddress returned NULL");
        if (get_ctx(&ctx) != CUDA_SUCCESS || !ctx) return fail(GAE_ERR_CUDA, "no current CUDA context");
        g_static_ws_ptr[dev] = p;
        g_static_ws_ctx[dev] = ctx;
    }
    *out = g_static_ws_ptr[dev];
    return GAE_OK;
}

}  // namespace

extern "C" gae_status gae_layer_fwd_static(const gae_layer_args *a, const gae_layer_weights *w,
                                           void *stream) {
    if (!a) return fail(GAE_ERR_INVALID_ARG, "args is NULL");
    if (a->batch < 1 || a->seq < 1 || a->d_model < 1 || a->d_ff < 1)
        return fail(GAE_ERR_INVALID_ARG, "invalid layer shape");
    if (a->batch > ((int64_t)1 << 31) / a->seq)
        return fail(GAE_ERR_INVALID_ARG, "batch*seq beyond 2^31 tokens");
    const LayerWs L = layer_ws(a->batch * a->seq, a->d_model, a->d_ff);
    if (!L.ok) return fail(GAE_ERR_INVALID_ARG, "layer shape too large (workspace size overflows)");
    const size_t need = L.total;
    if (need > kStaticLayerWsBytes)
        return fail(GAE_ERR_UNSUPPORTED,
                    "gae_layer_fwd_static: this shape needs %zu bytes of workspace, above the "
                    "fixed %zu-byte static workspace; use gae_layer_fwd with a caller workspace",
                    need, kStaticLayerWsBytes);
    void *ws = nullptr;
    gae_status s = static_ws_address(&ws);
    if (s != GAE_OK) return s;
    gae_layer_args b = *a;
    b.workspace = ws;
    b.workspace_bytes = kStaticLayerWsBytes;
    if ((s = check_layer(&b, w)) != GAE_OK) return s;
    return layer_once(&b, w, b.x, b.out, static_cast<cudaStream_t>(stream));
}
