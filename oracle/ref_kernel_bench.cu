// Test and comparison infrastructure only: builds the reference's published
// attention chain (cuda_src/waller_kernel_bench.cu:40-290: per tile a cuBLAS
// fp16 GEMM for the scores, an online-softmax kernel, a cuBLAS GEMM for P*V
// and an output-update kernel; the source of its 174.4 TFLOPS figure) from
// the reference tree where it lies (the file is included, not copied) into
// oracle/_ref/, with one extern "C" entry that runs the reference's own
// run_benchmark().  Never linked by the product library.
#ifndef GAE_REF_KERNEL_BENCH_SRC
#error "define GAE_REF_KERNEL_BENCH_SRC as the path of the reference's waller_kernel_bench.cu"
#endif
#define main gae_ref_kernel_bench_unused_main
#include GAE_REF_KERNEL_BENCH_SRC
#undef main

// One sequence (one head) of seq_len x head_dim fp16 through the reference's
// tiled chain with tile size `tile`, `iters` timed iterations.  Returns the
// reference's own figure: TFLOPS counted as 4 * seq_len^2 * head_dim per
// iteration (:272), whatever the causal tile loop skips.
extern "C" float ref_kernel_bench_tflops(int seq_len, int head_dim, int tile, int iters) {
    return run_benchmark(seq_len, head_dim, tile, iters, false);
}
