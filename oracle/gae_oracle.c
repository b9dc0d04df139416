/*
 * gae_oracle.c -- CPU restatement of the Geodesic Attention Engine's reference
 * path (the pure-Rust crate `ate`, the files under rust_src/src).
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels of the gae-b200 library.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg load it.  The product library never links it and
 * has no CPU fallback.
 *
 * Parity pin: the reference's Rust toolchain is absent here, so the Rust crate
 * cannot be run.  The restatement is pinned instead against every known-answer
 * test the reference ships for this path (tests/validation.rs:6-163), which the
 * Python tests replay through this library (tests/test_oracle.py).
 *
 * Semantics kept from the reference, with the exact operation order:
 *   - sequential f32 dot product, then `* scale`  (waller_operator.rs:29-31)
 *   - branchy OnlineSoftmax::update               (online_softmax.rs:28-35)
 *   - correction exp(old_max - new_max) applied only when old_max != -inf
 *                                                 (waller_operator.rs:38-43)
 *   - weight exp(score - max), acc += weight * v  (waller_operator.rs:46-49)
 *   - final acc / sum (a division)                (waller_operator.rs:53-56)
 * Build with -O3 -ffp-contract=off and no fast-math so that every f32
 * operation rounds as Rust's IEEE f32 arithmetic does; expf/tanhf/sqrtf come
 * from the same libm that Rust's f32 methods call on Linux.
 *
 * Extensions (documented, not in the reference): a `causal` flag (causal=0
 * lets j run over all keys with the identical recurrence), batched (B,H)
 * layouts with query/key position offsets, a log-sum-exp output, the int8
 * logit path with per-row scales, and a pre-norm GPT-2 layer composed from the
 * restated primitives.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* OnlineSoftmax  (rust_src/src/online_softmax.rs:5-41)                       */
/* ------------------------------------------------------------------------ */
typedef struct { float max; float sum; } ora_online_softmax;

void ora_online_softmax_init(ora_online_softmax *s) { s->max = -INFINITY; s->sum = 0.0f; }

/* online_softmax.rs:28-35 */
void ora_online_softmax_update(ora_online_softmax *s, float score) {
    if (score > s->max) {
        s->sum = s->sum * expf(s->max - score) + 1.0f;
        s->max = score;
    } else {
        s->sum += expf(score - s->max);
    }
}

/* online_softmax.rs:38-40 */
float ora_online_softmax_probability(const ora_online_softmax *s, float score) {
    return expf(score - s->max) / s->sum;
}

/* ------------------------------------------------------------------------ */
/* WelfordState  (rust_src/src/welford.rs:20-55)                              */
/* ------------------------------------------------------------------------ */
typedef struct { float mean; float m2; uint32_t count; } ora_welford;

void ora_welford_init(ora_welford *w) { w->mean = 0.0f; w->m2 = 0.0f; w->count = 0; }

/* welford.rs:27-33 */
void ora_welford_update(ora_welford *w, float x) {
    w->count += 1;
    float delta = x - w->mean;
    w->mean += delta / (float)w->count;
    float delta2 = x - w->mean;
    w->m2 += delta * delta2;
}

/* welford.rs:36-38 (population variance, 0 below two samples) */
float ora_welford_variance(const ora_welford *w) {
    return w->count < 2 ? 0.0f : w->m2 / (float)w->count;
}

/* welford.rs:41-43 */
float ora_welford_std(const ora_welford *w, float eps) {
    return sqrtf(ora_welford_variance(w) + eps);
}

/* welford.rs:46-55 (Chan merge) */
void ora_welford_merge(const ora_welford *a, const ora_welford *b, ora_welford *out) {
    uint32_t count = a->count + b->count;
    if (count == 0) { ora_welford_init(out); return; }
    float delta = b->mean - a->mean;
    float mean = a->mean + delta * (float)b->count / (float)count;
    float m2 = a->m2 + b->m2 + delta * delta * (float)a->count * (float)b->count / (float)count;
    out->mean = mean; out->m2 = m2; out->count = count;
}

/* ------------------------------------------------------------------------ */
/* Activations  (rust_src/src/activations.rs:5-19)                            */
/* ------------------------------------------------------------------------ */
/* activations.rs:5-7: the tanh form, 0.5x(1+tanh(sqrt(2/pi)(x+0.044715x^3))).
 * x.powi(3) is evaluated as (x*x)*x; sqrt(2/pi) is an f32 sqrt of the f32
 * quotient 2/PI. */
float ora_gelu(float x) {
    const float c = sqrtf(2.0f / 3.14159265358979323846f);
    float x3 = (x * x) * x;
    return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x3)));
}
/* activations.rs:11-13 */
float ora_silu(float x) { return x / (1.0f + expf(-x)); }
/* activations.rs:17-19 */
float ora_relu(float x) { return x > 0.0f ? x : 0.0f; }

/* ------------------------------------------------------------------------ */
/* LayerNorm  (rust_src/src/layernorm.rs:6-47)                                */
/* ------------------------------------------------------------------------ */
/* layernorm.rs:6-17 */
void ora_layernorm(const float *in, const float *gamma, const float *beta,
                   size_t n, float eps, float *out) {
    ora_welford w; ora_welford_init(&w);
    for (size_t i = 0; i < n; ++i) ora_welford_update(&w, in[i]);
    float mean = w.mean, sd = ora_welford_std(&w, eps);
    for (size_t i = 0; i < n; ++i) out[i] = (in[i] - mean) / sd * gamma[i] + beta[i];
}

/* layernorm.rs:20-47 */
void ora_layernorm_batched(const float *in, const float *gamma, const float *beta,
                           size_t batch, size_t hidden, float eps, float *out) {
    #pragma omp parallel for schedule(static)
    for (size_t b = 0; b < batch; ++b)
        ora_layernorm(in + b * hidden, gamma, beta, hidden, eps, out + b * hidden);
}

/* ------------------------------------------------------------------------ */
/* MLP  (rust_src/src/mlp.rs:7-73)                                            */
/* ------------------------------------------------------------------------ */
/* mlp.rs:7-36: W1 [hidden, mlp], W2 [mlp, hidden], row-major; the bias seeds
 * the sum. */
void ora_mlp_block(const float *in, const float *w1, const float *b1,
                   const float *w2, const float *b2, size_t hidden, size_t mlp,
                   float *out) {
    float *mid = (float *)malloc(mlp * sizeof(float));
    for (size_t i = 0; i < mlp; ++i) {
        float s = b1[i];
        for (size_t j = 0; j < hidden; ++j) s += in[j] * w1[j * mlp + i];
        mid[i] = ora_gelu(s);
    }
    for (size_t i = 0; i < hidden; ++i) {
        float s = b2[i];
        for (size_t j = 0; j < mlp; ++j) s += mid[j] * w2[j * hidden + i];
        out[i] = s;
    }
    free(mid);
}

/* mlp.rs:39-73: MLP, + residual, Welford LayerNorm. */
void ora_fused_mlp_layernorm(const float *in, const float *residual,
                             const float *w1, const float *b1,
                             const float *w2, const float *b2,
                             const float *gamma, const float *beta,
                             size_t hidden, size_t mlp, float eps, float *out) {
    float *m = (float *)malloc(hidden * sizeof(float));
    ora_mlp_block(in, w1, b1, w2, b2, hidden, mlp, m);
    for (size_t i = 0; i < hidden; ++i) m[i] = m[i] + residual[i];
    ora_welford w; ora_welford_init(&w);
    for (size_t i = 0; i < hidden; ++i) ora_welford_update(&w, m[i]);
    float mean = w.mean, sd = ora_welford_std(&w, eps);
    for (size_t i = 0; i < hidden; ++i) out[i] = (m[i] - mean) / sd * gamma[i] + beta[i];
    free(m);
}

/* transformer.rs:124-134: y = W[m,n] x */
static void ora_matvec(const float *w, const float *x, size_t m, size_t n, float *y) {
    for (size_t i = 0; i < m; ++i) {
        float s = 0.0f;
        for (size_t j = 0; j < n; ++j) s += w[i * n + j] * x[j];
        y[i] = s;
    }
}

/* transformer.rs:87-120: the reference's demo forward (LN1 -> Wv -> Wo + res
 * -> fused MLP + LN, no cross-token attention).  Weights as in
 * TransformerBlock: wv/wo [h,h] as W[out,in]; w1 [h,m]; w2 [m,h]. */
void ora_transformer_block_forward(const float *input, size_t seq_len, size_t h, size_t m,
                                   float eps, const float *wv, const float *wo,
                                   const float *ln1_g, const float *ln1_b,
                                   const float *w1, const float *b1,
                                   const float *w2, const float *b2,
                                   const float *ln2_g, const float *ln2_b, float *out) {
    #pragma omp parallel for schedule(static)
    for (size_t pos = 0; pos < seq_len; ++pos) {
        const float *row = input + pos * h;
        float *normed = (float *)malloc(h * sizeof(float));
        float *v = (float *)malloc(h * sizeof(float));
        float *proj = (float *)malloc(h * sizeof(float));
        ora_layernorm(row, ln1_g, ln1_b, h, eps, normed);
        ora_matvec(wv, normed, h, h, v);
        ora_matvec(wo, v, h, h, proj);
        for (size_t i = 0; i < h; ++i) proj[i] = proj[i] + row[i];
        ora_fused_mlp_layernorm(proj, proj, w1, b1, w2, b2, ln2_g, ln2_b, h, m, eps,
                                out + pos * h);
        free(normed); free(v); free(proj);
    }
}

/* ------------------------------------------------------------------------ */
/* Waller operator  (rust_src/src/waller_operator.rs:8-117)                   */
/* ------------------------------------------------------------------------ */
/* One query row of waller_operator.rs:17-57.  Keys j in [0, jend).  Returns
 * the final softmax state so callers can form a log-sum-exp. */
static ora_online_softmax waller_row(const float *qrow, const float *k, const float *v,
                                     size_t kstride, size_t jend, size_t d, float scale,
                                     float *acc, float *out_row) {
    ora_online_softmax sm; ora_online_softmax_init(&sm);
    for (size_t c = 0; c < d; ++c) acc[c] = 0.0f;
    for (size_t j = 0; j < jend; ++j) {
        const float *krow = k + j * kstride;
        const float *vrow = v + j * kstride;
        float dot = 0.0f;
        for (size_t c = 0; c < d; ++c) dot += qrow[c] * krow[c];
        float score = dot * scale;
        float old_max = sm.max;
        ora_online_softmax_update(&sm, score);
        if (old_max != -INFINITY) {
            float corr = expf(old_max - sm.max);
            for (size_t c = 0; c < d; ++c) acc[c] *= corr;
        }
        float weight = expf(score - sm.max);
        for (size_t c = 0; c < d; ++c) acc[c] += weight * vrow[c];
    }
    for (size_t c = 0; c < d; ++c) out_row[c] = acc[c] / sm.sum;
    return sm;
}

/* waller_operator.rs:8-59 with the causal flag (causal=1 is the reference). */
void ora_waller_operator(const float *q, const float *k, const float *v,
                         size_t seq_len, size_t head_dim, float scale, int causal,
                         float *out) {
    float *acc = (float *)malloc(head_dim * sizeof(float));
    for (size_t i = 0; i < seq_len; ++i)
        waller_row(q + i * head_dim, k, v, head_dim, causal ? i + 1 : seq_len, head_dim,
                   scale, acc, out + i * head_dim);
    free(acc);
}

/* waller_operator.rs:62-109: the same body, rows in parallel (rayon there,
 * OpenMP here).  Dynamic scheduling because row i costs i+1 pairs. */
void ora_waller_operator_parallel(const float *q, const float *k, const float *v,
                                  size_t seq_len, size_t head_dim, float scale, int causal,
                                  float *out) {
    #pragma omp parallel
    {
        float *acc = (float *)malloc(head_dim * sizeof(float));
        #pragma omp for schedule(dynamic, 16)
        for (size_t i = 0; i < seq_len; ++i)
            waller_row(q + i * head_dim, k, v, head_dim, causal ? i + 1 : seq_len, head_dim,
                       scale, acc, out + i * head_dim);
        free(acc);
    }
}

/* standard_attention.rs:13-65: materialised scores, -inf mask, row softmax,
 * weighted sum.  causal=0 fills every score (extension). */
void ora_standard_attention(const float *q, const float *k, const float *v,
                            size_t n, size_t d, float scale, int causal, float *out) {
    float *scores = (float *)malloc(n * n * sizeof(float));
    for (size_t i = 0; i < n; ++i)
        for (size_t j = 0; j < n; ++j) {
            if (!causal || j <= i) {
                float dot = 0.0f;
                for (size_t c = 0; c < d; ++c) dot += q[i * d + c] * k[j * d + c];
                scores[i * n + j] = dot * scale;
            } else {
                scores[i * n + j] = -INFINITY;
            }
        }
    for (size_t i = 0; i < n; ++i) {
        float *row = scores + i * n;
        float mx = -INFINITY;
        for (size_t j = 0; j < n; ++j) mx = fmaxf(mx, row[j]);
        float sum = 0.0f;
        for (size_t j = 0; j < n; ++j) { row[j] = expf(row[j] - mx); sum += row[j]; }
        for (size_t j = 0; j < n; ++j) row[j] /= sum;
    }
    for (size_t i = 0; i < n * d; ++i) out[i] = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        size_t jend = causal ? i + 1 : n;
        for (size_t j = 0; j < jend; ++j) {
            float w = scores[i * n + j];
            for (size_t c = 0; c < d; ++c) out[i * d + c] += w * v[j * d + c];
        }
    }
    free(scores);
}

/* ------------------------------------------------------------------------ */
/* Batched extension used by the bf16 / ring parity tests.                    */
/* Q [B,H,Nq,d], K/V [B,H,Nkv,d], O [B,H,Nq,d] contiguous fp32 (bf16 inputs   */
/* are widened by the caller).  Query row r sits at absolute position         */
/* q_offset + r, key column c at kv_offset + c; with causal=1 key c is seen   */
/* iff kv_offset + c <= q_offset + r.  lse (natural log, [B,H,Nq]) may be     */
/* NULL; a row that sees no key gets out=0 and lse=-inf.  Only rows listed    */
/* in `rows` (or all rows when rows==NULL) are computed.                      */
/* ------------------------------------------------------------------------ */
void ora_attention_batched(const float *q, const float *k, const float *v,
                           size_t B, size_t H, size_t nq, size_t nkv, size_t d,
                           float scale, int causal, long long q_offset, long long kv_offset,
                           const int64_t *rows, size_t nrows, float *out, float *lse) {
    size_t per_head = rows ? nrows : nq;
    size_t total = B * H * per_head;
    #pragma omp parallel
    {
        float *acc = (float *)malloc(d * sizeof(float));
        #pragma omp for schedule(dynamic, 8)
        for (size_t t = 0; t < total; ++t) {
            size_t bh = t / per_head, ri = t % per_head;
            size_t r = rows ? (size_t)rows[ri] : ri;
            const float *qh = q + (bh * nq + r) * d;
            const float *kh = k + bh * nkv * d;
            const float *vh = v + bh * nkv * d;
            float *orow = out + (bh * nq + r) * d;
            long long jend = (long long)nkv;
            if (causal) {
                long long lim = q_offset + (long long)r - kv_offset + 1;
                if (lim < jend) jend = lim;
                if (jend < 0) jend = 0;
            }
            if (jend == 0) {
                for (size_t c = 0; c < d; ++c) orow[c] = 0.0f;
                if (lse) lse[bh * nq + r] = -INFINITY;
                continue;
            }
            ora_online_softmax sm = waller_row(qh, kh, vh, d, (size_t)jend, d, scale, acc, orow);
            if (lse) lse[bh * nq + r] = sm.max + logf(sm.sum);
        }
        free(acc);
    }
}

/* Merge of two partial results over disjoint key sets, by log-sum-exp:
 * o = (e^(l1-m) o1 + e^(l2-m) o2) / (e^(l1-m) + e^(l2-m)), lse = m + log(...).
 * Same algebra as the reference's block merge of (max, sum, acc) states
 * (cuda_src/waller_operator_v2.cu:120-142). rows x d. In place into o1/l1. */
void ora_lse_merge(float *o1, float *l1, const float *o2, const float *l2,
                   size_t rows, size_t d) {
    #pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
        float a = l1[r], b = l2[r];
        float m = a > b ? a : b;
        if (m == -INFINITY) continue;
        float wa = expf(a - m), wb = expf(b - m);
        float s = wa + wb;
        for (size_t c = 0; c < d; ++c)
            o1[r * d + c] = (wa * o1[r * d + c] + wb * o2[r * d + c]) / s;
        l1[r] = m + logf(s);
    }
}

/* ------------------------------------------------------------------------ */
/* INT8 path (extension for the int8 configuration).                          */
/* ------------------------------------------------------------------------ */
/* Per-row symmetric quantisation: scale = max|x| / 127, q = rint(x / scale)
 * (round half to even), clamped to [-127, 127]; an all-zero row gets scale 0
 * and q = 0. */
void ora_quantize_rows_int8(const float *x, size_t rows, size_t d, int8_t *q, float *scale) {
    for (size_t r = 0; r < rows; ++r) {
        float mx = 0.0f;
        for (size_t c = 0; c < d; ++c) { float a = fabsf(x[r * d + c]); if (a > mx) mx = a; }
        float s = mx / 127.0f;
        scale[r] = s;
        for (size_t c = 0; c < d; ++c) {
            float v = (s > 0.0f) ? rintf(x[r * d + c] / s) : 0.0f;
            if (v > 127.0f) v = 127.0f;
            if (v < -127.0f) v = -127.0f;
            q[r * d + c] = (int8_t)v;
        }
    }
}

/* Exact int32 logits L[i][j] = sum_c qi8[i][c] * ki8[j][c] (the reference's
 * dot_int8, cuda_src/waller_operator_int8.cu:13-24).  Per (b,h) slices. */
void ora_int8_logits(const int8_t *q, const int8_t *k, size_t BH, size_t nq, size_t nkv,
                     size_t d, int32_t *out) {
    #pragma omp parallel for collapse(2) schedule(static)
    for (size_t bh = 0; bh < BH; ++bh)
        for (size_t i = 0; i < nq; ++i) {
            const int8_t *qr = q + (bh * nq + i) * d;
            for (size_t j = 0; j < nkv; ++j) {
                const int8_t *kr = k + (bh * nkv + j) * d;
                int32_t acc = 0;
                for (size_t c = 0; c < d; ++c) acc += (int32_t)qr[c] * (int32_t)kr[c];
                out[(bh * nq + i) * nkv + j] = acc;
            }
        }
}

/* INT8 attention: score = (float)logit * (sq[i] * sk[j]) * scale, then the
 * Waller recurrence with fp32 V (bf16 values widened). */
void ora_attention_int8(const int8_t *q, const int8_t *k, const float *sq, const float *sk,
                        const float *v, size_t BH, size_t n, size_t d, float scale,
                        int causal, const int64_t *rows, size_t nrows, float *out) {
    size_t per_head = rows ? nrows : n;
    #pragma omp parallel
    {
        float *acc = (float *)malloc(d * sizeof(float));
        #pragma omp for schedule(dynamic, 8)
        for (size_t t = 0; t < BH * per_head; ++t) {
            size_t bh = t / per_head, ri = t % per_head;
            size_t i = rows ? (size_t)rows[ri] : ri;
            const int8_t *qr = q + (bh * n + i) * d;
            size_t jend = causal ? i + 1 : n;
            ora_online_softmax sm; ora_online_softmax_init(&sm);
            for (size_t c = 0; c < d; ++c) acc[c] = 0.0f;
            for (size_t j = 0; j < jend; ++j) {
                const int8_t *kr = k + (bh * n + j) * d;
                const float *vr = v + (bh * n + j) * d;
                int32_t dot = 0;
                for (size_t c = 0; c < d; ++c) dot += (int32_t)qr[c] * (int32_t)kr[c];
                float score = (float)dot * (sq[bh * n + i] * sk[bh * n + j]) * scale;
                float old_max = sm.max;
                ora_online_softmax_update(&sm, score);
                if (old_max != -INFINITY) {
                    float corr = expf(old_max - sm.max);
                    for (size_t c = 0; c < d; ++c) acc[c] *= corr;
                }
                float w = expf(score - sm.max);
                for (size_t c = 0; c < d; ++c) acc[c] += w * vr[c];
            }
            float *orow = out + (bh * n + i) * d;
            for (size_t c = 0; c < d; ++c) orow[c] = acc[c] / sm.sum;
        }
        free(acc);
    }
}

/* ------------------------------------------------------------------------ */
/* Pre-norm GPT-2 layer composed from the restated primitives (extension for  */
/* the fused-layer configuration).  x [T, D] with T = B * S tokens; weights   */
/* in [in, out] row-major like mlp.rs's W1: Wqkv [D, 3D], Wproj [D, D],       */
/* Wfc [D, F], Wfc2 [F, D].  The qkv columns are [q | k | v], head h at       */
/* columns h*hd .. h*hd+hd-1 of each third.  When round_bf16 != 0 every       */
/* tensor the GPU stores between kernels is rounded to bf16 at the same point */
/* (LN outputs, qkv, attention output, residual stream, GELU output, layer    */
/* output), so the two paths differ only by fp32 summation order.            */
/* ------------------------------------------------------------------------ */
static float bf16_round(float x) {
    uint32_t u; memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) return x;       /* inf / nan */
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    u &= 0xffff0000u;
    float r; memcpy(&r, &u, 4);
    return r;
}

float ora_bf16_round(float x) { return bf16_round(x); }

static void gemm_bias(const float *x, const float *w, const float *b, size_t T, size_t K,
                      size_t N, float *y) {
    #pragma omp parallel for schedule(static)
    for (size_t t = 0; t < T; ++t) {
        float *yr = y + t * N;
        for (size_t n = 0; n < N; ++n) yr[n] = 0.0f;
        for (size_t kk = 0; kk < K; ++kk) {
            float xv = x[t * K + kk];
            const float *wr = w + kk * N;
            for (size_t n = 0; n < N; ++n) yr[n] += xv * wr[n];
        }
        for (size_t n = 0; n < N; ++n) yr[n] += b[n];
    }
}

void ora_gpt2_layer(const float *x, size_t Bsz, size_t S, size_t D, size_t nh, size_t F,
                    float eps, const float *ln1_g, const float *ln1_b,
                    const float *wqkv, const float *bqkv, const float *wproj,
                    const float *bproj, const float *ln2_g, const float *ln2_b,
                    const float *wfc, const float *bfc, const float *wfc2,
                    const float *bfc2, int round_bf16, float *out) {
    size_t T = Bsz * S, hd = D / nh;
    float *ln = (float *)malloc(T * D * sizeof(float));
    float *qkv = (float *)malloc(T * 3 * D * sizeof(float));
    float *att = (float *)malloc(T * D * sizeof(float));
    float *x1 = (float *)malloc(T * D * sizeof(float));
    float *hid = (float *)malloc(T * F * sizeof(float));
    float *tmp = (float *)malloc(T * (D > F ? D : F) * sizeof(float));
#define RND(p, n) do { if (round_bf16) for (size_t _i = 0; _i < (n); ++_i) (p)[_i] = bf16_round((p)[_i]); } while (0)
    ora_layernorm_batched(x, ln1_g, ln1_b, T, D, eps, ln);
    RND(ln, T * D);
    gemm_bias(ln, wqkv, bqkv, T, D, 3 * D, qkv);
    RND(qkv, T * 3 * D);
    float scale = 1.0f / sqrtf((float)hd);
    #pragma omp parallel
    {
        float *qh = (float *)malloc(S * hd * sizeof(float));
        float *kh = (float *)malloc(S * hd * sizeof(float));
        float *vh = (float *)malloc(S * hd * sizeof(float));
        float *oh = (float *)malloc(S * hd * sizeof(float));
        float *acc = (float *)malloc(hd * sizeof(float));
        #pragma omp for schedule(static)
        for (size_t bh = 0; bh < Bsz * nh; ++bh) {
            size_t b = bh / nh, h = bh % nh;
            for (size_t s = 0; s < S; ++s)
                for (size_t c = 0; c < hd; ++c) {
                    const float *r = qkv + ((b * S + s) * 3 * D);
                    qh[s * hd + c] = r[h * hd + c];
                    kh[s * hd + c] = r[D + h * hd + c];
                    vh[s * hd + c] = r[2 * D + h * hd + c];
                }
            for (size_t i = 0; i < S; ++i)
                waller_row(qh + i * hd, kh, vh, hd, i + 1, hd, scale, acc, oh + i * hd);
            for (size_t s = 0; s < S; ++s)
                for (size_t c = 0; c < hd; ++c)
                    att[(b * S + s) * D + h * hd + c] = oh[s * hd + c];
        }
        free(qh); free(kh); free(vh); free(oh); free(acc);
    }
    RND(att, T * D);
    gemm_bias(att, wproj, bproj, T, D, D, tmp);
    for (size_t i = 0; i < T * D; ++i) x1[i] = x[i] + tmp[i];
    RND(x1, T * D);
    ora_layernorm_batched(x1, ln2_g, ln2_b, T, D, eps, ln);
    RND(ln, T * D);
    gemm_bias(ln, wfc, bfc, T, D, F, hid);
    for (size_t i = 0; i < T * F; ++i) hid[i] = ora_gelu(hid[i]);
    RND(hid, T * F);
    gemm_bias(hid, wfc2, bfc2, T, F, D, tmp);
    for (size_t i = 0; i < T * D; ++i) out[i] = x1[i] + tmp[i];
    RND(out, T * D);
#undef RND
    free(ln); free(qkv); free(att); free(x1); free(hid); free(tmp);
}

int ora_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Sets the OpenMP thread count of later parallel regions (the CPU baseline
 * uses every host core whatever OMP_NUM_THREADS a launcher exported). */
void ora_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------------------ */
/* Fused "symphony" layer (cuda_src/waller_fused_layer.cu:64-247): one token  */
/* through identity-Q int8 causal attention, a gated residual, RMSNorm, an    */
/* MLP with a selectable activation, a gated residual and RMSNorm.  tf holds  */
/* the TuningFork fields (waller_fused_layer.cu:23-32) in order: attn_scale,  */
/* attn_temperature, residual_alpha, residual_beta, norm_eps, mlp_gate,       */
/* output_scale; act is activation_type (0 GELU-tanh, 1 SiLU, 2 ReLU^2).      */
/* input/output [n, d] fp32, k/v int8 [n, d], w_up [d, 4d], w_down [4d, d].   */
/* ------------------------------------------------------------------------ */
static float sym_act(float x, int type) {  /* waller_fused_layer.cu:35-46 */
    switch (type) {
        case 0: return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
        case 1: return x / (1.0f + expf(-x));
        case 2: return x > 0.0f ? x * x : 0.0f;
        default: return x;
    }
}

static void sym_rmsnorm(float *x, const float *w, size_t d, float eps) {  /* :49-60 */
    float ss = 0.0f;
    for (size_t i = 0; i < d; ++i) ss += x[i] * x[i];
    float scale = 1.0f / sqrtf(ss / (float)d + eps);
    for (size_t i = 0; i < d; ++i) x[i] = x[i] * scale * w[i];
}

void ora_symphony_layer(const float *input, const int8_t *k, const int8_t *v, const float *w_up,
                        const float *w_down, const float *n1, const float *n2, size_t n, size_t d,
                        const float *tf, int act, float *out) {
    const float attn_scale = tf[0], temp = tf[1], alpha = tf[2], beta = tf[3], eps = tf[4];
    const float gate = tf[5], oscale = tf[6];
    const size_t m = 4 * d;
    #pragma omp parallel
    {
        float *state = (float *)malloc(d * sizeof(float));
        float *res = (float *)malloc(d * sizeof(float));
        float *acc = (float *)malloc(d * sizeof(float));
        float *hid = (float *)malloc(m * sizeof(float));
        int8_t *q = (int8_t *)malloc(d);
        #pragma omp for schedule(dynamic, 16)
        for (size_t row = 0; row < n; ++row) {
            for (size_t c = 0; c < d; ++c) { state[c] = input[row * d + c]; res[c] = state[c]; }
            /* :113-118 identity projection, quantised by truncation */
            for (size_t c = 0; c < d; ++c) q[c] = (int8_t)fmaxf(-127.0f, fminf(127.0f, state[c] * 127.0f));
            /* :123-185 causal attention, per-key online softmax */
            float mx = -INFINITY, sum = 0.0f;
            for (size_t c = 0; c < d; ++c) acc[c] = 0.0f;
            for (size_t j = 0; j <= row; ++j) {
                int32_t dot = 0;
                for (size_t c = 0; c < d; ++c) dot += (int32_t)q[c] * (int32_t)k[j * d + c];
                float score = (float)dot * attn_scale / temp;
                float old = mx;
                mx = fmaxf(mx, score);
                float resc = expf(old - mx);
                sum = sum * resc + expf(score - mx);
                float w = expf(score - mx);
                for (size_t c = 0; c < d; ++c) acc[c] = acc[c] * resc + w * (float)v[j * d + c];
            }
            float inv = 1.0f / sum;
            /* :190-194 */
            for (size_t c = 0; c < d; ++c) state[c] = res[c] * alpha + acc[c] * inv;
            sym_rmsnorm(state, n1, d, eps);
            for (size_t c = 0; c < d; ++c) res[c] = state[c];
            /* :207-229 */
            for (size_t i = 0; i < m; ++i) {
                float s = 0.0f;
                for (size_t c = 0; c < d; ++c) s += state[c] * w_up[c * m + i];
                hid[i] = sym_act(s, act);
            }
            for (size_t c = 0; c < d; ++c) {
                float s = 0.0f;
                for (size_t i = 0; i < m; ++i) s += hid[i] * w_down[i * d + c];
                acc[c] = s * gate;
            }
            /* :234-246 */
            for (size_t c = 0; c < d; ++c) state[c] = res[c] * beta + acc[c];
            sym_rmsnorm(state, n2, d, eps);
            for (size_t c = 0; c < d; ++c) out[row * d + c] = state[c] * oscale;
        }
        free(state); free(res); free(acc); free(hid); free(q);
    }
}

/* Attention backward (an extension: the reference is inference-only).  The
 * standard gradients of O = softmax(scale * Q K^T) V per (batch, head) slice,
 * computed directly from the definition in double precision:
 *   P = softmax rows (causal: keys j <= i), dV = P^T dO, dP = dO V^T,
 *   dS = P o (dP - rowsum(dO o O)) with O recomputed here, dQ = scale dS K,
 *   dK = scale dS^T Q.
 * q, dout: [BH, nq, d]; k, v: [BH, nkv, d]; outputs likewise (float). */
void ora_attention_bwd(const float *q, const float *k, const float *v, const float *dout, size_t BH,
                       size_t nq, size_t nkv, size_t d, float scale, int causal, float *dq, float *dk,
                       float *dv) {
    #pragma omp parallel for schedule(dynamic, 1)
    for (size_t bh = 0; bh < BH; ++bh) {
        const float *Q = q + bh * nq * d, *K = k + bh * nkv * d, *V = v + bh * nkv * d;
        const float *G = dout + bh * nq * d;
        float *dQ = dq + bh * nq * d, *dK = dk + bh * nkv * d, *dV = dv + bh * nkv * d;
        double *P = (double *)malloc(nkv * sizeof(double));
        double *dKa = (double *)calloc(nkv * d, sizeof(double));
        double *dVa = (double *)calloc(nkv * d, sizeof(double));
        double *o = (double *)malloc(d * sizeof(double));
        for (size_t i = 0; i < nq; ++i) {
            const size_t nk = causal ? (i + 1 < nkv ? i + 1 : nkv) : nkv;
            double mx = -INFINITY;
            for (size_t j = 0; j < nk; ++j) {
                double s = 0.0;
                for (size_t c = 0; c < d; ++c) s += (double)Q[i * d + c] * (double)K[j * d + c];
                P[j] = s * scale;
                if (P[j] > mx) mx = P[j];
            }
            double sum = 0.0;
            for (size_t j = 0; j < nk; ++j) { P[j] = exp(P[j] - mx); sum += P[j]; }
            for (size_t c = 0; c < d; ++c) o[c] = 0.0;
            for (size_t j = 0; j < nk; ++j) {
                P[j] /= sum;
                for (size_t c = 0; c < d; ++c) o[c] += P[j] * (double)V[j * d + c];
            }
            double delta = 0.0;
            for (size_t c = 0; c < d; ++c) delta += o[c] * (double)G[i * d + c];
            double *dqa = (double *)calloc(d, sizeof(double));
            for (size_t j = 0; j < nk; ++j) {
                double dp = 0.0;
                for (size_t c = 0; c < d; ++c) {
                    dp += (double)G[i * d + c] * (double)V[j * d + c];
                    dVa[j * d + c] += P[j] * (double)G[i * d + c];
                }
                const double ds = P[j] * (dp - delta);
                for (size_t c = 0; c < d; ++c) {
                    dqa[c] += ds * (double)K[j * d + c];
                    dKa[j * d + c] += ds * (double)Q[i * d + c];
                }
            }
            for (size_t c = 0; c < d; ++c) dQ[i * d + c] = (float)(dqa[c] * scale);
            free(dqa);
        }
        for (size_t x = 0; x < nkv * d; ++x) {
            dK[x] = (float)(dKa[x] * scale);
            dV[x] = (float)dVa[x];
        }
        free(P); free(dKa); free(dVa); free(o);
    }
}
