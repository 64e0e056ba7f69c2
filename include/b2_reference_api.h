// b2_reference_api.h — the reference's own C++ launch API, served by the B200 kernels.
//
// Same names, parameter lists and pointer conventions as the reference headers, so its
// engine, tests and benchmarks link against this library unchanged:
//   run_decode_attn            kernels/decode/13_decode_attn.cuh:192-199
//   run_quantize_fp32_to_int8  kernels/quantization/14_int8_gemm.cuh:20-23
//   run_int8_gemm              kernels/quantization/14_int8_gemm.cuh:28-33
//   run_int8_gemm_bias         kernels/quantization/14_int8_gemm.cuh:39-45
//   run_int8_gemm_bias_gelu    kernels/quantization/14_int8_gemm.cuh:48-54
//   run_int8_gemm_bias_residual kernels/quantization/14_int8_gemm.cuh:57-64
//   DA_MAX_SPLITS              kernels/decode/13_decode_attn.cuh:12 (callers size the workspace with it)
//   I8Epilogue                 kernels/quantization/14_int8_gemm.cuh:36
//
// All pointers are device pointers; launches go to the legacy default stream. These
// return void like the reference's, but do not fail silently: the status of the last call
// is b2_last_status() (include/b2decode.h), and unsupported shapes (e.g. a GQA group of 3,
// which the reference ignores, 13_decode_attn.cu:306) are reported there.
//
// run_decode_attn's workspace keeps the reference's size, [B, H_q, DA_MAX_SPLITS, d+2]
// floats; it needs no initialisation.
#pragma once
#include <cstdint>
#include "b2decode.h"

#define DA_MAX_SPLITS 16

enum class I8Epilogue { Plain, BiasOnly, BiasGELU, BiasResidual };

void run_decode_attn(int B, int H_q, int H_kv, int d, const float* Q, const float* k_cache, const float* v_cache,
                     const int* block_table, const int* context_lens, int max_context_len, int block_size,
                     int num_blocks_per_seq, float* O, float* workspace);

void run_quantize_fp32_to_int8(int rows, int cols, const float* input, int32_t* output_packed, float* scales);

void run_int8_gemm(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed, const float* scale_A,
                   const float* scale_B, float* C);

void run_int8_gemm_bias(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed,
                        const float* scale_A, const float* scale_B, const float* bias, float* C);

void run_int8_gemm_bias_gelu(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed,
                             const float* scale_A, const float* scale_B, const float* bias, float* C);

void run_int8_gemm_bias_residual(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed,
                                 const float* scale_A, const float* scale_B, const float* bias,
                                 const float* residual, float* C);
