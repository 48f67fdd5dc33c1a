// ref_cpu_harness.cu — exposes the reference's own host-side oracle functions with C linkage.
// It includes the reference test sources unmodified (their main() renamed) from the reference
// tree; nothing is copied. Test infrastructure only.
#define main fence_ref_test_gemv_main
#include "tests/test_gemv_q6k.cu"
#undef main


extern "C" {
// cpu_gemv_q6k, tests/test_gemv_q6k.cu:117-128
void ref_cpu_gemv_q6k(const void* W, const void* x, double* y, int M, int K) {
    cpu_gemv_q6k(static_cast<const block_q6_K*>(W), static_cast<const __half*>(x), y, M, K);
}
// cpu_q6k_dot_block, tests/test_gemv_q6k.cu:78-114
double ref_cpu_q6k_dot_block(const void* blk, const void* x) {
    return cpu_q6k_dot_block(*static_cast<const block_q6_K*>(blk), static_cast<const __half*>(x));
}
// set_q6, tests/test_gemv_q6k.cu:41-74 (the inverse layout map)
void ref_set_q6(void* blk, int i, int val) { set_q6(*static_cast<block_q6_K*>(blk), i, val); }
}
