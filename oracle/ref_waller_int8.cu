// Test infrastructure only: builds the reference's own INT8 Waller kernel
// (cuda_src/waller_operator_int8.cu:27-68, compiled from the reference tree
// where it lies; the file is included, not copied) into oracle/_ref/ with one
// extern "C" launcher, so that tests can pin the oracle's INT8 restatement and
// this library's INT8 attention against it.  Never linked by the product
// library.  The reference's main() is renamed out of the way; the kernel is
// launched as its benchmark does (:102-106: 256 threads a block, one a row).
#include <cstdint>
#ifndef GAE_REF_WALLER_INT8_SRC
#error "define GAE_REF_WALLER_INT8_SRC as the path of the reference's waller_operator_int8.cu"
#endif
#define main gae_ref_waller_int8_unused_main
#include GAE_REF_WALLER_INT8_SRC
#undef main

// Device pointers, [seq_len, head_dim] int8 (head_dim <= 128), fp32 output;
// score = dot * qk_scale, value = v / v_scale.  Returns the cudaError_t.
extern "C" int ref_waller_int8_fwd(const int8_t *q, const int8_t *k, const int8_t *v, float *out, int seq_len,
                                   int head_dim, float qk_scale, float v_scale, void *stream) {
    const int block = 256, grid = (seq_len + block - 1) / block;
    waller_operator_int8_kernel<<<grid, block, 0, (cudaStream_t)stream>>>(q, k, v, out, seq_len, head_dim, qk_scale,
                                                                          v_scale);
    return (int)cudaGetLastError();
}
