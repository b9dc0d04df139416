// Test infrastructure only: builds the reference's head_dim-128 and -256
// fused layer kernels (cuda_src/waller_fused_realistic.cu:26-148
// waller_fused_128 and :151-274 waller_fused_256, the symphony layer of
// waller_fused_layer.cu at HEAD_DIM 128 / MLP 512 and 256 / 1024, compiled
// from the reference tree where it lies; the file is included, not copied)
// into oracle/_ref/ with one extern "C" launcher each, so that tests can pin
// the CPU restatement ora_symphony_layer and gae_symphony_fwd at those widths.
// Never linked by the product library.
//
// The reference's main() is renamed out of the way; the kernel is launched
// as its benchmark does (:329-334: grid ceil(N/32) x 32 threads).
#include <cstdint>
#ifndef GAE_REF_REALISTIC_SRC
#error "define GAE_REF_REALISTIC_SRC as the path of the reference's waller_fused_realistic.cu"
#endif
#define main gae_ref_realistic_unused_main
#include GAE_REF_REALISTIC_SRC
#undef main

// tf = {attn_scale, temperature, alpha, beta, eps, mlp_gate, output_scale}.
// Device pointers; returns the cudaError_t.
extern "C" int ref_symphony128_fwd(const int8_t *k, const int8_t *v, const float *w_up, const float *w_down,
                                   const float *n1, const float *n2, const float *input, float *output,
                                   int seq_len, const float *tf, int act, void *stream) {
    TuningFork t;
    t.attn_scale = tf[0];
    t.attn_temperature = tf[1];
    t.residual_alpha = tf[2];
    t.residual_beta = tf[3];
    t.norm_eps = tf[4];
    t.activation_type = act;
    t.mlp_gate = tf[5];
    t.output_scale = tf[6];
    const int block = 32, grid = (seq_len + block - 1) / block;
    waller_fused_128<<<grid, block, 0, (cudaStream_t)stream>>>(k, v, w_up, w_down, n1, n2, input, output,
                                                               seq_len, t);
    return (int)cudaGetLastError();
}

extern "C" int ref_symphony256_fwd(const int8_t *k, const int8_t *v, const float *w_up, const float *w_down,
                                   const float *n1, const float *n2, const float *input, float *output,
                                   int seq_len, const float *tf, int act, void *stream) {
    TuningFork t;
    t.attn_scale = tf[0];
    t.attn_temperature = tf[1];
    t.residual_alpha = tf[2];
    t.residual_beta = tf[3];
    t.norm_eps = tf[4];
    t.activation_type = act;
    t.mlp_gate = tf[5];
    t.output_scale = tf[6];
    const int block = 32, grid = (seq_len + block - 1) / block;
    waller_fused_256<<<grid, block, 0, (cudaStream_t)stream>>>(k, v, w_up, w_down, n1, n2, input, output,
                                                               seq_len, t);
    return (int)cudaGetLastError();
}
