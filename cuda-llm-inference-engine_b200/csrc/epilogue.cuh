// Dequantisation epilogue of the INT8 GEMM, shared by the fused GEMM epilogue and the
// tensor-parallel path (which applies it after an int32 all-reduce).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include "b2decode.h"

namespace b2 {

__device__ __forceinline__ float gelu_tanh(float v) {
    // 0.5 v (1 + tanh(sqrt(2/pi) (v + 0.044715 v^3))), operation order of the reference
    // epilogue (kernels/quantization/14_int8_gemm.cu:158-160) with its contraction.
    const float x3 = __fmul_rn(__fmul_rn(v, v), v);
    const float inner = __fmul_rn(0.7978845608f, __fmaf_rn(0.044715f, x3, v));
    return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(inner)));
}

template <int EPI>
__device__ __forceinline__ float epilogue(int32_t acc, float sa, float sb, float bias, float res) {
    const float t = __fmul_rn(__int2float_rn(acc), sa);
    if constexpr (EPI == B2_EPI_PLAIN) {
        return __fmul_rn(t, sb);
    } else {
        const float v = __fmaf_rn(t, sb, bias);
        if constexpr (EPI == B2_EPI_BIAS) return v;
        if constexpr (EPI == B2_EPI_BIAS_GELU) return gelu_tanh(v);
        return __fadd_rn(v, res);
    }
}

}  // namespace b2
