// Exposes the reference's own code, compiled from its sources where they lie, to the
// tests as an oracle (test infrastructure only; built by oracle/build_ref.sh into
// oracle/_ref/libref.so):
//   - gqa_cpu_reference, the reference harness's CPU attention (tests/test_paged_attention.cu:138-179);
//   - run_decode_attn (K13), run_quantize_fp32_to_int8 and run_int8_gemm* (K14), and
//     run_paged_attn / run_gqa_paged_attn (K11/K12, the reference's GPU oracle for K13),
//     and run_layernorm (K15), built for sm_100a unchanged.
// Only the extern "C" ref_* symbols below are exported.
#include "tests/test_paged_attention.cu"  // from the reference tree (-I REF)
#include "decode/13_decode_attn.cuh"
#include "quantization/14_int8_gemm.cuh"
#include "layernorm/15_layernorm_residual.cuh"

#define REF_API extern "C" __attribute__((visibility("default")))

REF_API void ref_gqa_cpu_reference(int B, int H_q, int H_kv, int N, int d, const float* Q, const float* K,
                                   const float* V, float* O, int causal) {
    gqa_cpu_reference(B, H_q, H_kv, N, d, Q, K, V, O, causal != 0);
}

REF_API void ref_run_decode_attn(int B, int H_q, int H_kv, int d, const float* Q, const float* k_cache,
                                 const float* v_cache, const int* block_table, const int* context_lens,
                                 int max_context_len, int block_size, int num_blocks_per_seq, float* O,
                                 float* workspace) {
    run_decode_attn(B, H_q, H_kv, d, Q, k_cache, v_cache, block_table, context_lens, max_context_len, block_size,
                    num_blocks_per_seq, O, workspace);
}

REF_API void ref_run_gqa_paged_attn(int B, int H_q, int H_kv, int N, int d, const float* Q, const float* k_cache,
                                    const float* v_cache, const int* block_table, const int* context_lens,
                                    int max_context_len, int block_size, int num_blocks_per_seq, float* O,
                                    int causal) {
    run_gqa_paged_attn(B, H_q, H_kv, N, d, Q, k_cache, v_cache, block_table, context_lens, max_context_len,
                       block_size, num_blocks_per_seq, O, causal != 0);
}

REF_API void ref_run_quantize_fp32_to_int8(int rows, int cols, const float* input, int32_t* out, float* scales) {
    run_quantize_fp32_to_int8(rows, cols, input, out, scales);
}

REF_API void ref_run_int8_gemm(int M, int N, int K, const int32_t* A, const int32_t* BT, const float* sA,
                               const float* sB, const float* bias, const float* residual, float* C, int epi) {
    switch (epi) {
        case 0: run_int8_gemm(M, N, K, A, BT, sA, sB, C); break;
        case 1: run_int8_gemm_bias(M, N, K, A, BT, sA, sB, bias, C); break;
        case 2: run_int8_gemm_bias_gelu(M, N, K, A, BT, sA, sB, bias, C); break;
        default: run_int8_gemm_bias_residual(M, N, K, A, BT, sA, sB, bias, residual, C); break;
    }
}

REF_API void ref_run_layernorm(int rows, int cols, const float* x, const float* gamma, const float* beta, float* out,
                               float eps) {
    run_layernorm(rows, cols, x, gamma, beta, out, eps);
}

REF_API int ref_sync(void) { return (int)cudaDeviceSynchronize(); }
