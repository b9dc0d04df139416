// Test infrastructure only: builds the reference's own fp32 Waller operator
// kernels (cuda_src/waller_operator.cu:12-100, single head and multi-head,
// compiled from the reference tree where it lies; the file is included, not
// copied) into oracle/_ref/ with extern "C" launchers, so that tests can pin
// the CPU restatement and this library's attention paths against the
// reference's GPU kernel.  Never linked by the product library.
//
// The reference's main() is renamed out of the way; the kernels are launched
// as its benchmark does (:150-163: 256 threads a block, one thread a row).
#include <cstdint>
#ifndef GAE_REF_WALLER_SRC
#error "define GAE_REF_WALLER_SRC as the path of the reference's waller_operator.cu"
#endif
#define main gae_ref_waller_unused_main
#include GAE_REF_WALLER_SRC
#undef main

// Device pointers, [seq_len, head_dim] row-major (head_dim <= 128); returns
// the cudaError_t.
extern "C" int ref_waller_operator_fwd(const float *q, const float *k, const float *v, float *out,
                                       int seq_len, int head_dim, float scale, void *stream) {
    const int block = 256, grid = (seq_len + block - 1) / block;
    waller_operator_kernel<<<grid, block, 0, (cudaStream_t)stream>>>(q, k, v, out, seq_len, head_dim, scale);
    return (int)cudaGetLastError();
}

// [num_heads, seq_len, head_dim].
extern "C" int ref_waller_operator_multihead_fwd(const float *q, const float *k, const float *v, float *out,
                                                 int seq_len, int head_dim, int num_heads, float scale,
                                                 void *stream) {
    const int block = 256, grid = (seq_len * num_heads + block - 1) / block;
    waller_operator_multihead_kernel<<<grid, block, 0, (cudaStream_t)stream>>>(q, k, v, out, seq_len, head_dim,
                                                                               num_heads, scale);
    return (int)cudaGetLastError();
}
