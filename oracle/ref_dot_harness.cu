// ref_dot_harness.cu — exposes the hand-built golden blocks of the reference's Q6_K dot test
// (tests/test_q6k_dot.cu:242-332) and its fp64 host oracle cpu_q6k_dot (:41-86), included
// unmodified from the reference tree with main() renamed. Test infrastructure only.
#define main fence_ref_test_dot_main
#include "tests/test_q6k_dot.cu"
#undef main

extern "C" {
// the six hand-built cases of tests/test_q6k_dot.cu:242-332 and their fp64 expectation
int ref_dot_case(int idx, void* blk_out, void* x_out, double* expected) {
    TestCase tc;
    switch (idx) {
        case 0: tc = make_test_zero_centered(); break;
        case 1: tc = make_test_all_min(); break;
        case 2: tc = make_test_all_max(); break;
        case 3: tc = make_test_random(); break;
        case 4: tc = make_test_mixed_scales(); break;
        case 5: tc = make_test_single_subblock(); break;
        default: return -1;
    }
    memcpy(blk_out, &tc.blk, sizeof(block_q6_K));
    memcpy(x_out, tc.x_host, sizeof(tc.x_host));
    *expected = cpu_q6k_dot(tc.blk, tc.x_host);
    return 0;
}
const char* ref_dot_case_name(int idx) {
    static const char* names[6] = {"all_quants_32_zero_centered", "all_quants_0_minimum", "all_quants_63_maximum",
                                   "random_quants_uniform_x", "mixed_pos_neg_scales", "single_nonzero_subblock"};
    return (idx >= 0 && idx < 6) ? names[idx] : "";
}
}
