/*
 * gae.h -- C ABI of the gae-b200 library (libgae.so): the Geodesic Attention
 * Engine's fused "Waller" attention path, rebuilt for NVIDIA B200 (sm_100a).
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, never
 * throws or exits, and returns a gae_status.  On failure a thread-local detail
 * string is available from gae_last_error().  Entry points that take a
 * `stream` are asynchronous with respect to the host and ordered on that CUDA
 * stream (pass a cudaStream_t cast to void*, or NULL for the legacy default
 * stream).  The *_host entry points take host memory and are synchronous.
 *
 * Each declaration names the reference interface it replaces
 * (RegularJoe-CEO/Geodesic-Attention-Engine-GAE-, path:line inside that
 * project).  The reference crate `ate` panics on bad input; a Rust binding
 * keeps those semantics by turning a non-GAE_OK status back into a panic.
 */
#ifndef GAE_H_
#define GAE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GAE_API __attribute__((visibility("default")))
#else
#define GAE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    GAE_OK = 0,
    GAE_ERR_INVALID_ARG = 1,  /* bad shape, stride, alignment or pointer      */
    GAE_ERR_UNSUPPORTED = 2,  /* valid request this build has no kernel for   */
    GAE_ERR_CUDA = 3,         /* a CUDA runtime/driver call failed            */
    GAE_ERR_OOM = 4,          /* device allocation failed (host entry points) */
    GAE_ERR_COMM = 5,         /* ring transport failure                       */
    GAE_ERR_TIMEOUT = 6       /* a bounded device-side wait gave up           */
} gae_status;

typedef enum {
    GAE_DTYPE_F32 = 0,
    GAE_DTYPE_BF16 = 1,
    GAE_DTYPE_F16 = 2
} gae_dtype;

/* Human-readable name of a status code (static string). */
GAE_API const char *gae_status_string(gae_status s);

/* Copies the calling thread's last error detail into buf (NUL-terminated,
 * truncated to n bytes) and returns the status it was recorded with. */
GAE_API gae_status gae_last_error(char *buf, size_t n);

/* Library version, "major.minor.patch". */
GAE_API const char *gae_version(void);

/* Synchronises the current device and reports whether any kernel of this
 * library recorded a device-side failure (a bounded wait that ran out) since
 * the last reset.  reset != 0 clears the record.  GAE_OK or GAE_ERR_TIMEOUT. */
GAE_API gae_status gae_device_status(int reset);

/* ------------------------------------------------------------------------
 * Host-memory drop-ins for the Rust crate's attention functions.
 * Layout as in the reference: q, k, v, out are [seq_len, head_dim] fp32
 * row-major, one head.  Computes out[i] = sum_j softmax_j(scale*<q_i,k_j>) v_j
 * over j <= i (causal != 0, the reference's only mode) or over all j
 * (causal == 0).  fp32 CUDA-core kernel, fp32 throughout.  head_dim <= 256.
 * ---------------------------------------------------------------------- */

/* replaces ate::waller_operator, rust_src/src/waller_operator.rs:8-15 */
GAE_API gae_status gae_waller_operator_f32_host(const float *q, const float *k, const float *v,
                                        size_t seq_len, size_t head_dim, float scale,
                                        int causal, float *out);

/* replaces ate::waller_operator_parallel, rust_src/src/waller_operator.rs:63-70
 * (same result; the GPU runs all rows in parallel either way) */
GAE_API gae_status gae_waller_operator_parallel_f32_host(const float *q, const float *k,
                                                 const float *v, size_t seq_len,
                                                 size_t head_dim, float scale, int causal,
                                                 float *out);

/* replaces ate::standard_attention, rust_src/src/standard_attention.rs:13-20.
 * The reference materialises the N x N scores; this entry point returns the
 * same softmax attention through the fused streaming kernel (no N x N
 * buffer), which the reference's own test pins as equal within 1e-4
 * (tests/validation.rs:147-163). */
GAE_API gae_status gae_standard_attention_f32_host(const float *q, const float *k, const float *v,
                                           size_t seq_len, size_t head_dim, float scale,
                                           int causal, float *out);

/* ------------------------------------------------------------------------
 * The crate's fp32 layer functions, computed in the crate's own order.
 * Each output element is one sequential f32 sum in increasing index order
 * with no fused multiply-add, and LayerNorm uses the crate's single-pass
 * Welford statistics, so sums, statistics and normalisation match the
 * crate's f32 results bit for bit; GELU's tanh may differ in the last place.
 * Host entry points take host slices as the crate does and are synchronous
 * (they allocate device memory for the call).  `tokens` rows are processed
 * independently; the crate's own call is tokens = 1.  Any widths.
 * ---------------------------------------------------------------------- */

/* replaces ate::layernorm, rust_src/src/layernorm.rs:6-17 (one row of n) */
GAE_API gae_status gae_layernorm_f32_host(const float *input, const float *gamma, const float *beta,
                                          size_t n, float eps, float *out);

/* replaces ate::layernorm_batched, rust_src/src/layernorm.rs:20-47 */
GAE_API gae_status gae_layernorm_batched_f32_host(const float *input, const float *gamma,
                                                  const float *beta, size_t batch, size_t hidden,
                                                  float eps, float *out);

/* replaces ate::mlp_block, rust_src/src/mlp.rs:7-36: gelu(x @ W1 + b1) @ W2 + b2,
 * W1 [hidden_dim, mlp_dim], W2 [mlp_dim, hidden_dim] row-major (the crate's
 * layouts); input/out [tokens, hidden_dim]. */
GAE_API gae_status gae_mlp_block_f32_host(const float *input, const float *w1, const float *b1,
                                          const float *w2, const float *b2, size_t hidden_dim,
                                          size_t mlp_dim, size_t tokens, float *out);

/* replaces ate::fused_mlp_layernorm, rust_src/src/mlp.rs:39-73:
 * LayerNorm(mlp_block(input) + residual) per token. */
GAE_API gae_status gae_fused_mlp_layernorm_f32_host(const float *input, const float *residual,
                                                    const float *w1, const float *b1,
                                                    const float *w2, const float *b2,
                                                    const float *gamma, const float *beta,
                                                    size_t hidden_dim, size_t mlp_dim, float eps,
                                                    size_t tokens, float *out);

/* The weights and config of ate::TransformerBlock (rust_src/src/transformer.rs:
 * 9-33): wq/wk/wv/wo [hidden, hidden] as W[out, in] (wq and wk are unused by
 * the crate's forward and may be NULL), w1 [hidden, mlp], w2 [mlp, hidden]. */
typedef struct {
    const float *wq, *wk, *wv, *wo;
    const float *ln1_gamma, *ln1_beta;
    const float *w1, *b1;
    const float *w2, *b2;
    const float *ln2_gamma, *ln2_beta;
    size_t hidden_dim, num_heads, head_dim, mlp_dim;
    float eps;
} gae_transformer_block_f32;

/* replaces ate::TransformerBlock::forward, rust_src/src/transformer.rs:87-120:
 * per token LN1 -> Wv -> Wo + input -> fused_mlp_layernorm(r1, r1) (the
 * crate's forward has no cross-token attention).  input/out [seq_len, hidden]. */
GAE_API gae_status gae_transformer_block_forward_f32_host(const gae_transformer_block_f32 *block,
                                                          const float *input, size_t seq_len,
                                                          float *out);

/* Device-pointer forms of the two kernels above (stream-ordered):
 * y[M, N] = epi(init + sum_j x[M, j] * W(j, n)), init = bias[n] or 0 (bias
 * NULL), W(j, n) = w[j*N + n] when w_in_major (the crate's W1/W2) else
 * w[n*K + j] (the crate's matvec, transformer.rs:124-134); epilogue 0 none,
 * 1 GELU (activations.rs:5-7), 2 + res[M, N].  And the Welford LayerNorm of
 * rows [rows, d]. */
GAE_API gae_status gae_crate_linear_f32(const float *x, const float *w, const float *bias,
                                        const float *res, float *y, int64_t M, int64_t N, int64_t K,
                                        int w_in_major, int epilogue, void *stream);
GAE_API gae_status gae_crate_layernorm_f32(const float *x, const float *gamma, const float *beta,
                                           float *y, int64_t rows, int64_t d, float eps, void *stream);

/* ------------------------------------------------------------------------
 * Device-pointer attention (the reference's CUDA Waller kernels:
 * cuda_src/waller_operator.cu:12-100 fp32, cuda_src/waller_kernel_bench.cu:
 * 164-290 fp16 tiles, cuda_src/bench_tma.cu:152-429 TMA/wgmma).
 *
 * Q [batch, heads, seq_q, head_dim], K/V [batch, heads, seq_kv, head_dim],
 * O like Q, addressed through element strides {batch, head, seq}; the
 * head_dim stride is 1.  lse (optional, fp32, contiguous [batch, heads,
 * seq_q]) receives the natural-log log-sum-exp of each row's scaled scores,
 * -inf for a row that sees no key (its O row is 0).
 *
 * Query row r is at absolute position q_offset + r and key column c at
 * kv_offset + c; with causal != 0 key c is visible to row r iff
 * kv_offset + c <= q_offset + r.  The offsets let a sequence-parallel caller
 * run one block of a ring step.
 *
 * dtype BF16/F16: tcgen05 tensor-core kernel, head_dim 64 or 128, fp32
 * softmax and accumulation, O in the input dtype; all strides multiples of 8
 * elements and pointers 16-byte aligned (TMA rules).
 * dtype F32: CUDA-core fp32 kernel, any head_dim <= 256.
 * ---------------------------------------------------------------------- */
typedef struct {
    const void *q;
    const void *k;
    const void *v;
    void *o;
    float *lse;                 /* may be NULL */
    int64_t batch, heads, seq_q, seq_kv, head_dim;
    int64_t q_stride[3];        /* element strides: batch, head, seq */
    int64_t k_stride[3];
    int64_t v_stride[3];
    int64_t o_stride[3];
    gae_dtype dtype;
    int causal;
    float scale;                /* usually 1/sqrt(head_dim) */
    int64_t q_offset;
    int64_t kv_offset;
} gae_attn_args;

GAE_API gae_status gae_attn_fwd(const gae_attn_args *args, void *stream);

/* ------------------------------------------------------------------------
 * Sequence-parallel ring attention over P GPUs (no reference counterpart:
 * the reference has no multi-GPU path; this is its long-sequence caller).
 * One process or thread per GPU; each rank holds a contiguous shard
 * [B, H, S, D] of one sequence of N = P*S tokens (rank r owns positions
 * [r*S, (r+1)*S)) and receives the exact attention output of its queries
 * against the whole sequence, with the natural-log LSE if requested.
 *
 * Transport: an NCCL communicator (libnccl.so.2 is loaded at run time).
 * K/V blocks travel rank r -> r+1 by ncclSend/ncclRecv on an internal
 * stream, overlapped with the attention kernels on the caller's stream;
 * partial results are merged by log-sum-exp (gae_lse_merge's algebra) in
 * fp32.  With GAE_RING_ZIGZAG and causal != 0 the shards are re-dealt so that
 * rank r computes on chunks r and 2P-1-r of 2P (equal work per rank and
 * step) and the output is dealt back.  Remote blocks land in this GPU's
 * memory before any kernel reads them.
 *
 * The context owns a device arena (grown on demand; about 10x the shard's
 * bytes) and a non-blocking communicator.  Waits on the communicator and,
 * when timeout_s > 0, the completion of each gae_ring_attn_fwd are bounded
 * by timeout_s: on expiry the communicator is aborted, the call returns
 * GAE_ERR_TIMEOUT (GAE_ERR_COMM for an NCCL error) and the context refuses
 * further work.  With timeout_s <= 0 the call returns once everything is
 * enqueued (asynchronous, unbounded).  A context is used by one host thread
 * at a time, on the device current at its creation.
 * ---------------------------------------------------------------------- */
#define GAE_RING_UNIQUE_ID_BYTES 128
enum { GAE_RING_ZIGZAG = 0, GAE_RING_CONTIGUOUS = 1 };
typedef struct gae_ring_ctx gae_ring_ctx;

/* A fresh NCCL unique id (GAE_RING_UNIQUE_ID_BYTES bytes) that one rank
 * creates and every rank passes to gae_ring_ctx_create. */
GAE_API gae_status gae_ring_unique_id(void *unique_id);

/* Joins the P-rank communicator of unique_id as `rank` (collective: every
 * rank calls it).  With world == 1 no communicator is made (unique_id is
 * not read, NCCL is not loaded). */
GAE_API gae_status gae_ring_ctx_create(const void *unique_id, int rank, int world, double timeout_s,
                                       gae_ring_ctx **ctx);

/* Uses a caller-owned ncclComm_t (passed as void*; not destroyed by
 * gae_ring_ctx_destroy). */
GAE_API gae_status gae_ring_ctx_create_from_comm(void *nccl_comm, double timeout_s, gae_ring_ctx **ctx);

/* args: this rank's shards as for gae_attn_fwd (bf16 or f16, head_dim 64 or
 * 128, seq_q == seq_kv = S, offsets 0); balance GAE_RING_ZIGZAG (causal; S
 * even) or GAE_RING_CONTIGUOUS.  Collective: every rank calls it with the
 * same shapes.  With one rank it is one gae_attn_fwd launch. */
GAE_API gae_status gae_ring_attn_fwd(gae_ring_ctx *ctx, const gae_attn_args *args, int balance, void *stream);

GAE_API gae_status gae_ring_ctx_destroy(gae_ring_ctx *ctx);

/* ------------------------------------------------------------------------
 * Attention backward: dQ, dK, dV of the exact attention computed by
 * gae_attn_fwd, from Q, K, V, the forward output O, the output gradient dO
 * and the forward's LSE (natural log, [batch*heads, seq_q] as gae_attn_fwd
 * writes it).  No reference counterpart: the reference crate is
 * inference-only; this is the training-side caller of its operator
 * (P = softmax(scale * Q K^T), dV = P^T dO, dS = P o (dO V^T - rowsum(dO o O)),
 * dQ = scale * dS K, dK = scale * dS^T Q).
 * bf16 or f16, head_dim 64 or 128; causal requires seq_q == seq_kv (the
 * forward's mask with zero offsets).  Every pointer 16-byte aligned and every
 * stride a multiple of 8 elements.  `workspace`: device memory of at least
 * gae_attn_bwd_workspace_bytes(batch, heads, seq_q, head_dim) bytes (fp32 dQ
 * accumulator and the per-row dO.O sums).
 * ---------------------------------------------------------------------- */
typedef struct {
    const void *q;
    const void *k;
    const void *v;
    const void *o;
    const void *dout;
    const float *lse;
    void *dq;
    void *dk;
    void *dv;
    int64_t batch, heads, seq_q, seq_kv, head_dim;
    int64_t q_stride[3];        /* element strides: batch, head, seq */
    int64_t k_stride[3];
    int64_t v_stride[3];
    int64_t o_stride[3];
    int64_t do_stride[3];
    int64_t dq_stride[3];
    int64_t dk_stride[3];
    int64_t dv_stride[3];
    gae_dtype dtype;
    int causal;
    float scale;
    void *workspace;
    size_t workspace_bytes;
} gae_attn_bwd_args;

GAE_API size_t gae_attn_bwd_workspace_bytes(int64_t batch, int64_t heads, int64_t seq_q, int64_t head_dim);

GAE_API gae_status gae_attn_bwd(const gae_attn_bwd_args *args, void *stream);

/* ------------------------------------------------------------------------
 * INT8 attention (replaces cuda_src/waller_operator_int8.cu:27-67,
 * waller_operator_int8_tc.cu:38-87, waller_operator_int8_tiled.cu:15-189).
 * q, k: int8 [batch*heads, seq, head_dim] contiguous, with fp32 per-row
 * dequantisation scales q_scale/k_scale [batch*heads, seq]; v, o: bf16
 * [batch*heads, seq, head_dim].  logit(i,j) = int32 dot(q_i, k_j) computed
 * exactly (tcgen05 kind::i8, int32 accumulation);
 * score = logit * q_scale[i] * k_scale[j] * scale; softmax and P*V in fp32
 * accumulation with P rounded to bf16.  head_dim 64 or 128.
 * ---------------------------------------------------------------------- */
typedef struct {
    const int8_t *q;
    const int8_t *k;
    const float *q_scale;
    const float *k_scale;
    const void *v;              /* bf16 */
    void *o;                    /* bf16 */
    float *lse;                 /* may be NULL */
    int64_t batch_heads, seq, head_dim;
    int causal;
    float scale;
} gae_attn_int8_args;

GAE_API gae_status gae_attn_int8_fwd(const gae_attn_int8_args *args, void *stream);

/* Writes the exact int32 logits L[bh][i][j] = sum_c q[bh][i][c]*k[bh][j][c]
 * through the same tcgen05 kind::i8 tiles the attention kernel uses, for
 * bit-exact verification (the reference's dot_int8,
 * cuda_src/waller_operator_int8.cu:13-24).  logits: int32
 * [batch_heads, seq_q, seq_kv]. */
GAE_API gae_status gae_int8_logits(const int8_t *q, const int8_t *k, int64_t batch_heads,
                           int64_t seq_q, int64_t seq_kv, int64_t head_dim,
                           int32_t *logits, void *stream);

/* Per-row symmetric int8 quantisation: scale = max|x|/127, q = rint(x/scale)
 * clamped to +-127 (an all-zero row gets scale 0).  x: bf16 or fp32
 * [rows, d] contiguous.  (Extension: the reference quantises on the host with
 * a per-tensor 127 scale, cuda_src/waller_operator_int8.cu:99-100.) */
GAE_API gae_status gae_quantize_rows_int8(const void *x, gae_dtype dtype, int64_t rows, int64_t d,
                                  int8_t *q, float *scale, void *stream);

/* ------------------------------------------------------------------------
 * Log-sum-exp merge of two partial attention results over disjoint key sets
 * (the (max, sum, acc) merge of cuda_src/waller_operator_v2.cu:120-142,
 * restated on normalised outputs): in place
 *   m = max(lse_acc, lse_part); a = e^(lse_acc-m); b = e^(lse_part-m)
 *   o_acc = (a*o_acc + b*o_part)/(a+b);  lse_acc = m + log(a+b).
 * o_acc ([rows, head_dim], row stride o_acc_row_stride elements, type
 * acc_dtype) and o_part (row stride o_part_row_stride, type part_dtype) may
 * differ in type, e.g. an fp32 accumulator fed bf16 partials by a ring of
 * sequence-parallel steps; lse: fp32 [rows] contiguous.  Rows with both
 * lse = -inf are left as is.
 * ---------------------------------------------------------------------- */
GAE_API gae_status gae_lse_merge(void *o_acc, float *lse_acc, const void *o_part,
                         const float *lse_part, int64_t rows, int64_t head_dim,
                         int64_t o_acc_row_stride, int64_t o_part_row_stride,
                         gae_dtype acc_dtype, gae_dtype part_dtype, void *stream);

/* ------------------------------------------------------------------------
 * Fused pre-norm transformer layer (replaces the fused "symphony" layer,
 * cuda_src/waller_fused_layer.cu:64-247, and the API of
 * ate::TransformerBlock::forward, rust_src/src/transformer.rs:87-120, for a
 * real causal attention layer at GPT-2 shape):
 *   h   = LN1(x); qkv = h @ Wqkv + bqkv; a = causal_attention(qkv)
 *   x1  = x + a @ Wproj + bproj
 *   out = x1 + gelu_tanh(LN2(x1) @ Wfc + bfc) @ Wfc2 + bfc2
 * Activations bf16 [tokens = batch*seq, d_model] contiguous; weights bf16
 * stored [out, in] row-major (K-major for the tensor cores); biases and LN
 * parameters fp32.  `workspace` is caller-provided device memory of at least
 * gae_layer_workspace_bytes(...) bytes.  x and out may alias.
 * ---------------------------------------------------------------------- */
typedef struct {
    const void *ln1_gamma, *ln1_beta;   /* fp32 [d_model] */
    const void *w_qkv, *b_qkv;          /* bf16 [3*d_model, d_model], fp32 [3*d_model] */
    const void *w_proj, *b_proj;        /* bf16 [d_model, d_model],  fp32 [d_model] */
    const void *ln2_gamma, *ln2_beta;   /* fp32 [d_model] */
    const void *w_fc, *b_fc;            /* bf16 [d_ff, d_model],     fp32 [d_ff] */
    const void *w_fc2, *b_fc2;          /* bf16 [d_model, d_ff],     fp32 [d_model] */
} gae_layer_weights;

typedef struct {
    const void *x;              /* bf16 [batch*seq, d_model] */
    void *out;                  /* bf16 [batch*seq, d_model] */
    int64_t batch, seq, d_model, heads, d_ff;
    float eps;
    void *workspace;
    size_t workspace_bytes;
} gae_layer_args;

GAE_API size_t gae_layer_workspace_bytes(int64_t batch, int64_t seq, int64_t d_model, int64_t d_ff);

GAE_API gae_status gae_layer_fwd(const gae_layer_args *args, const gae_layer_weights *w, void *stream);

/* A stack of n_layers pre-norm layers applied in order (the GPT-2 stack);
 * ping-pongs between out and the workspace. */
GAE_API gae_status gae_layer_stack_fwd(const gae_layer_args *args, const gae_layer_weights *w,
                               int n_layers, void *stream);

/* One layer exactly as gae_layer_fwd, for callers that cannot allocate device
 * memory (allocator or memory-pool callbacks, plugins whose host owns every
 * device allocation, real-time paths where cudaMalloc may block).  No
 * counterpart in the reference.  The workspace fields of args are ignored: the
 * layer's scratch lives in a fixed 32 MiB device array inside libgae.so that
 * every GPU loading the library holds until exit.  Shapes whose
 * gae_layer_workspace_bytes exceeds 32 MiB (e.g. about 1980 tokens at GPT-2
 * small widths) return GAE_ERR_UNSUPPORTED.  Nothing is allocated; the first
 * call on a device looks up the array's device address (cudaGetSymbolAddress),
 * so make that first call before any stream capture; after a cudaDeviceReset
 * the next call looks it up again (make that call outside capture too).  Every call shares the one
 * array, which keeps the previous call's contents (the layer writes every
 * workspace byte it reads, so nothing needs clearing); calls that overlap on
 * the GPU (other streams, other threads) race on it and must be serialised by
 * the caller. */
GAE_API gae_status gae_layer_fwd_static(const gae_layer_args *args, const gae_layer_weights *w,
                                        void *stream);

/* One linear layer of the fused layer, exposed for callers and tests:
 * y[M, N] = x[M, K] @ w[N, K]^T + bias, then per `epilogue`: 0 nothing,
 * 1 tanh-GELU (rust_src/src/activations.rs:5-7), 2 + res[M, N].  bf16 x, w,
 * res, y (row-major, contiguous rows), fp32 bias (may be NULL); N % 256 == 0,
 * K % 64 == 0.  Replaces the matvecs of rust_src/src/mlp.rs:7-36 and
 * transformer.rs:124-134 with a tcgen05 GEMM. */
GAE_API gae_status gae_linear_fwd(const void *x, const void *w, const float *bias, const void *res,
                                  void *y, int64_t M, int64_t N, int64_t K, int epilogue, void *stream);

/* ------------------------------------------------------------------------
 * The reference's fused "symphony" layer (cuda_src/waller_fused_layer.cu:
 * 64-247; its knobs are the TuningFork struct, :23-32, mirrored field by
 * field): per token, Q = trunc(clamp(x*127, +-127)) (identity projection),
 * causal attention with int8 K and the integer values of int8 V,
 * score = dot * attn_scale / attn_temperature; state = x*residual_alpha +
 * attn -> RMSNorm(norm1_w, norm_eps) -> MLP (x @ w_up [d, 4d], activation
 * 0 GELU-tanh / 1 SiLU / 2 ReLU^2 / any other value the identity, as the
 * reference's `default:` branch, @ w_down [4d, d], * mlp_gate) ->
 * state*residual_beta + mlp -> RMSNorm(norm2_w) -> * output_scale.
 * input/output fp32 [seq_len, head_dim], k/v int8 [seq_len, head_dim], weights
 * fp32 row-major; head_dim 64 or 128 (tensor-core attention) or 256 (the
 * reference's waller_fused_256, cuda_src/waller_fused_realistic.cu:151-274;
 * attention on the CUDA cores in fp32); input, output, w_up, w_down and the
 * workspace 16-byte aligned.  `workspace`: device memory of at least
 * gae_symphony_workspace_bytes(seq_len, head_dim) bytes.
 * ---------------------------------------------------------------------- */
typedef struct {
    float attn_scale;
    float attn_temperature;
    float residual_alpha;
    float residual_beta;
    float norm_eps;
    int activation_type;
    float mlp_gate;
    float output_scale;
} gae_tuning_fork;

GAE_API size_t gae_symphony_workspace_bytes(int64_t seq_len, int64_t head_dim);

GAE_API gae_status gae_symphony_fwd(const float *input, const int8_t *k, const int8_t *v,
                                    const float *w_up, const float *w_down, const float *norm1_w,
                                    const float *norm2_w, int64_t seq_len, int64_t head_dim,
                                    const gae_tuning_fork *tuning, float *output, void *workspace,
                                    size_t workspace_bytes, void *stream);

/* Row LayerNorm with the reference's semantics (population variance, eps
 * inside the sqrt; rust_src/src/layernorm.rs:20-47): bf16 in/out, fp32
 * gamma/beta, optional fused residual add (res may be NULL: y = LN(x);
 * otherwise s = x + res is written to sum_out when non-NULL and y = LN(s)). */
GAE_API gae_status gae_layernorm_fwd(const void *x, const void *res, void *sum_out, void *y,
                             const float *gamma, const float *beta, int64_t rows,
                             int64_t d, float eps, void *stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* GAE_H_ */
