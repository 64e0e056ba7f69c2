// Row operations of the decode step, shared by the LayerNorm and quantiser kernels
// (engine_kernels.cu, int8_gemm.cu):
//   - ln_row_warp: LayerNorm, optionally fused with the per-row int8 quantiser, summing in
//     the order of the reference's 256-thread LayerNorm
//     (kernels/layernorm/15_layernorm_residual.cu:59-103) so the result is bit-identical;
//   - quant_row_warp: the per-row symmetric int8 quantiser
//     (kernels/quantization/14_int8_gemm.cu:22-58): scale = absmax / 127 (1 for an all-zero
//     row, IEEE division), q = clamp(rint(x * (1 / scale)), -128, 127), packed little-endian.
#pragma once
#include <cuda_bf16.h>
#include <cstdint>
#include "common.cuh"

namespace b2 {

// LayerNorm statistics from the row sums: mean = sum / cols, var = sumsq / cols - mean^2
// (one fused multiply-add), inv = rsqrtf(var + eps).
__device__ __forceinline__ void ln_stats(float sum, float sumsq, int cols, float eps, float& mean, float& inv) {
    const float n = (float)cols;
    mean = sum / n;
    const float var = fmaf(-mean, mean, sumsq / n);
    inv = rsqrtf(var + eps);
}

// Halving-tree sum of one value per thread of a 256-thread CTA in the reference LayerNorm's
// order (partial[t] += partial[t + s] for s = 128, 64, ..., 1; the total is partial[0]): strides
// 128, 64 and 32 through shared memory, then 16 .. 1 by shuffles within warp 0, whose lane 0
// pairing is the same tree. Every thread gets the total.
__device__ __forceinline__ float tree_sum256(float v, float* red) {
    const int t = threadIdx.x;
    red[t] = v;
    __syncthreads();
    if (t < 128) red[t] += red[t + 128];
    __syncthreads();
    if (t < 64) red[t] += red[t + 64];
    __syncthreads();
    if (t < 32) {
        float x = red[t] + red[t + 32];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x += __shfl_down_sync(0xffffffffu, x, o);
        if (t == 0) red[256] = x;
    }
    __syncthreads();
    const float total = red[256];
    __syncthreads();
    return total;
}

// LayerNorm (+ optional int8 quantisation) of one row of at most 256 * KC columns by one
// warp (16-byte aligned row and vectors). The reference's kernel has 256 threads; thread t
// sums columns t, t + 256, ... in order (squares with fused multiply-adds), then the 256
// partials are combined by a halving tree (partial[t] += partial[t + s], s = 128 .. 1).
// Here lane l loads float4s holding columns 4l + i + 128 h + 256 k (i < 4, h < 2, k < KC),
// i.e. the partials t = 4l + i + 128 h; stride 128 combines a lane's h = 0 and h = 1
// partials, strides 64 .. 4 pair lane l with lanes l + 16, 8, 4, 2, 1 (shuffles, same i),
// strides 2 and 1 combine lane 0's four i partials. q_row (nullable) [cols / 4] and
// *scale_out receive the quantised row; y_row / hi_row / lo_row (nullable) the normalised
// row in fp32 and as bf16 hi/lo halves. ln_row_regs takes the row already in registers
// (v[h][k] = columns 4 lane + 128 h + 256 k, zero past cols); ln_row_warp loads it first.
template <int KC>
__device__ __forceinline__ void ln_row_regs(float4 (&v)[2][KC], int cols, const float* __restrict__ gamma,
                                            const float* __restrict__ beta, float eps, int32_t* __restrict__ q_row,
                                            float* __restrict__ scale_out, float* __restrict__ y_row,
                                            __nv_bfloat16* __restrict__ hi_row, __nv_bfloat16* __restrict__ lo_row,
                                            int lane) {
    float ps[4] = {0.f, 0.f, 0.f, 0.f}, pq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        float s4[4] = {0.f, 0.f, 0.f, 0.f}, q4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < KC; ++k) {
            const int c = 4 * lane + 128 * h + 256 * k;
            if (c < cols) {
                const float t[4] = {v[h][k].x, v[h][k].y, v[h][k].z, v[h][k].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    s4[i] += t[i];
                    q4[i] = fmaf(t[i], t[i], q4[i]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // stride 128: partial t += partial t + 128
            ps[i] = h == 0 ? s4[i] : ps[i] + s4[i];
            pq[i] = h == 0 ? q4[i] : pq[i] + q4[i];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            ps[i] += __shfl_down_sync(0xffffffffu, ps[i], o);
            pq[i] += __shfl_down_sync(0xffffffffu, pq[i], o);
        }
    float s = (ps[0] + ps[2]) + (ps[1] + ps[3]);
    float ss = (pq[0] + pq[2]) + (pq[1] + pq[3]);
    s = __shfl_sync(0xffffffffu, s, 0);
    ss = __shfl_sync(0xffffffffu, ss, 0);
    float mean, inv;
    ln_stats(s, ss, cols, eps, mean, inv);
    float amax = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < KC; ++k) {
            const int c = 4 * lane + 128 * h + 256 * k;
            if (c < cols) {
                const float4 g = *reinterpret_cast<const float4*>(gamma + c);
                const float4 bb = *reinterpret_cast<const float4*>(beta + c);
                float4& t = v[h][k];
                t.x = fmaf(g.x * (t.x - mean), inv, bb.x);
                t.y = fmaf(g.y * (t.y - mean), inv, bb.y);
                t.z = fmaf(g.z * (t.z - mean), inv, bb.z);
                t.w = fmaf(g.w * (t.w - mean), inv, bb.w);
                amax = fmaxf(amax, fmaxf(fmaxf(fabsf(t.x), fabsf(t.y)), fmaxf(fabsf(t.z), fabsf(t.w))));
            }
        }
    if (!q_row) {  // plain LayerNorm (final ln_f feeding the vocab projection), fp32 and/or bf16 hi/lo
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int k = 0; k < KC; ++k) {
                const int c = 4 * lane + 128 * h + 256 * k;
                if (c >= cols) continue;
                if (y_row) *reinterpret_cast<float4*>(y_row + c) = v[h][k];
                if (hi_row) {
                    const float t[4] = {v[h][k].x, v[h][k].y, v[h][k].z, v[h][k].w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const __nv_bfloat16 hb = __float2bfloat16_rn(t[i]);
                        hi_row[c + i] = hb;
                        lo_row[c + i] = __float2bfloat16_rn(t[i] - __bfloat162float(hb));
                    }
                }
            }
        return;
    }
    amax = warp_max(amax);
    // quantiser semantics of kernels/quantization/14_int8_gemm.cu:36-58
    const float scale = amax > 0.f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    const float invs = __fdiv_rn(1.0f, scale);
    if (lane == 0) *scale_out = scale;
    int32_t* qr = q_row;
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < KC; ++k) {
            const int c = 4 * lane + 128 * h + 256 * k;
            if (c >= cols) continue;
            const float t[4] = {v[h][k].x, v[h][k].y, v[h][k].z, v[h][k].w};
            uint32_t packed = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float qf = fminf(fmaxf(rintf(__fmul_rn(t[i], invs)), -128.f), 127.f);
                packed |= (uint32_t)(uint8_t)(int8_t)(int)qf << (8 * i);
            }
            qr[c >> 2] = (int32_t)packed;
            if (y_row) *reinterpret_cast<float4*>(y_row + c) = v[h][k];
        }
}


// Loads the row (16-byte aligned) and runs ln_row_regs.
template <int KC>
__device__ __forceinline__ void ln_row_warp(const float* __restrict__ xr, int cols, const float* __restrict__ gamma,
                                            const float* __restrict__ beta, float eps, int32_t* __restrict__ q_row,
                                            float* __restrict__ scale_out, float* __restrict__ y_row,
                                            __nv_bfloat16* __restrict__ hi_row, __nv_bfloat16* __restrict__ lo_row,
                                            int lane) {
    float4 v[2][KC];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < KC; ++k) {
            const int c = 4 * lane + 128 * h + 256 * k;
            v[h][k] = c < cols ? *reinterpret_cast<const float4*>(xr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    ln_row_regs<KC>(v, cols, gamma, beta, eps, q_row, scale_out, y_row, hi_row, lo_row, lane);
}

// Per-row int8 quantisation of x[0, cols) by one warp (cols % 4 == 0, cols <= 128 * NV4,
// x 16-byte aligned): q_row [cols / 4] packed, *scale_out = the row's scale.
template <int NV4>
__device__ __forceinline__ void quant_row_warp(const float* __restrict__ x, int cols, int32_t* __restrict__ q_row,
                                               float* __restrict__ scale_out, int lane) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const int c4 = cols >> 2;
    float4 v[NV4];
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < NV4; ++k) {
        const int i = lane + 32 * k;
        v[k] = i < c4 ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[k].x), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w))));
    }
    amax = warp_max(amax);
    const float scale = amax > 0.f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, scale);
    if (lane == 0) *scale_out = scale;
#pragma unroll
    for (int k = 0; k < NV4; ++k) {
        const int i = lane + 32 * k;
        if (i < c4) {
            const float t[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
            uint32_t packed = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float q = fminf(fmaxf(rintf(__fmul_rn(t[j], inv)), -128.f), 127.f);
                packed |= (uint32_t)(uint8_t)(int8_t)(int)q << (8 * j);
            }
            q_row[i] = (int32_t)packed;
        }
    }
}

}  // namespace b2
