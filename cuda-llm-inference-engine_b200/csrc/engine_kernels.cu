// Small kernels of the batched GPT-2 decode step (one token per sequence per step).
//
// Reference semantics (mohith-suresh/CUDA-LLM-Inference-Engine):
//   embedding           kernels/layernorm/15_embed.cu:4-22      x = wte[id] + wpe[pos]
//   LayerNorm           kernels/layernorm/15_layernorm_residual.cu:59-103
//                       mean = sum/cols; var = sumsq/cols - mean^2; inv = rsqrtf(var + eps);
//                       y = gamma (x - mean) inv + beta
//   QKV split + KV write src/gpt2_engine.cu:292-346             Q||K||V per token; K,V to
//                       cache[((bt[pos/bs]*bs + pos%bs)*H + h)*dh + i]
//   vocab projection    src/gpt2_engine.cu:391-403              logits[v] = sum_k h[k] wte[v,k]
//   greedy sampling     src/sampler.cu:10-14                    argmax, lowest index on ties
// B200 changes: the step is batched over B sequences with per-sequence positions held on
// the device; LayerNorm is fused with the per-row int8 quantiser that follows it in every
// use (src/gpt2_engine.cu:460-463, 516-520); the QKV split is fused with the KV-cache write;
// the vocab projection is a tiled fp32 kernel over the whole batch fused with the argmax
// (64-bit atomicMax on an order-preserving key), so no logits leave the GPU; positions,
// context lengths and the next input token advance on the device, so a whole step is a
// fixed sequence of launches that a CUDA graph can replay.
#include "common.cuh"
#include "engine_kernels.cuh"
#include "epilogue.cuh"
#include <algorithm>
#include <cuda_bf16.h>

namespace b2 {

// ------------------------------------------------------------------ embedding
__global__ void embed_kernel(int d, const int* __restrict__ tokens, const int* __restrict__ pos,
                             const float* __restrict__ wte, const float* __restrict__ wpe, float* __restrict__ x,
                             int* __restrict__ ctx_lens, unsigned long long* __restrict__ argmax_keys) {
    griddep_wait();
    griddep_launch();
    const int b = blockIdx.x;
    const int tok = tokens[b];
    const int p = pos[b];
    const float* e = wte + (size_t)tok * d;
    const float* w = wpe + (size_t)p * d;
    float* o = x + (size_t)b * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) o[i] = e[i] + w[i];
    if (threadIdx.x == 0) {
        ctx_lens[b] = p + 1;     // attention of this step covers positions [0, p]
        argmax_keys[b] = 0ull;   // reset the greedy-sampling reduction for this step
    }
}

// ------------------------------------------------------------------ LayerNorm + int8 quantise
// One CTA per row; the row stays in registers (cols <= LNQ_THREADS * LNQ_MAX_PER_THREAD).
constexpr int LNQ_THREADS = 256;
constexpr int LNQ_MAX_PER_THREAD = 32;

__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < LNQ_THREADS / 32; ++w) t += red[w];
    __syncthreads();
    return t;
}

__global__ void __launch_bounds__(LNQ_THREADS)
ln_quant_kernel(int cols, const float* __restrict__ x, const float* __restrict__ gamma,
                const float* __restrict__ beta, float eps, int32_t* __restrict__ q_out,
                float* __restrict__ scale_out, float* __restrict__ y_out, __nv_bfloat16* __restrict__ y_hi,
                __nv_bfloat16* __restrict__ y_lo) {
    __shared__ float red[LNQ_THREADS / 32];
    griddep_wait();
    griddep_launch();
    const int row = blockIdx.x;
    const float* xr = x + (size_t)row * cols;
    float v[LNQ_MAX_PER_THREAD];
    float s = 0.f, ss = 0.f;
#pragma unroll
    for (int k = 0; k < LNQ_MAX_PER_THREAD; ++k) {
        const int c = threadIdx.x + k * LNQ_THREADS;
        v[k] = c < cols ? xr[c] : 0.f;
        s += v[k];
        ss = fmaf(v[k], v[k], ss);
    }
    const float mean = block_sum(s, red) / cols;
    const float var = block_sum(ss, red) / cols - mean * mean;
    const float inv = rsqrtf(var + eps);
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < LNQ_MAX_PER_THREAD; ++k) {
        const int c = threadIdx.x + k * LNQ_THREADS;
        if (c < cols) {
            v[k] = fmaf(gamma[c] * (v[k] - mean), inv, beta[c]);
            amax = fmaxf(amax, fabsf(v[k]));
        }
    }
    if (!q_out) {  // plain LayerNorm (final ln_f feeding the vocab projection), fp32 and/or bf16 hi/lo
#pragma unroll
        for (int k = 0; k < LNQ_MAX_PER_THREAD; ++k) {
            const int c = threadIdx.x + k * LNQ_THREADS;
            if (c < cols) {
                if (y_out) y_out[(size_t)row * cols + c] = v[k];
                if (y_hi) {
                    const __nv_bfloat16 h = __float2bfloat16_rn(v[k]);
                    y_hi[(size_t)row * cols + c] = h;
                    y_lo[(size_t)row * cols + c] = __float2bfloat16_rn(v[k] - __bfloat162float(h));
                }
            }
        }
        return;
    }
    amax = warp_max(amax);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int w = 1; w < LNQ_THREADS / 32; ++w) amax = fmaxf(amax, red[w]);
    // quantiser semantics of kernels/quantization/14_int8_gemm.cu:36-58
    const float scale = amax > 0.f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    const float invs = __fdiv_rn(1.0f, scale);
    if (threadIdx.x == 0) scale_out[row] = scale;
    int8_t* qb = reinterpret_cast<int8_t*>(q_out) + (size_t)row * cols;
#pragma unroll
    for (int k = 0; k < LNQ_MAX_PER_THREAD; ++k) {
        const int c = threadIdx.x + k * LNQ_THREADS;
        if (c < cols) {
            const float qf = fminf(fmaxf(rintf(__fmul_rn(v[k], invs)), -128.f), 127.f);
            qb[c] = (int8_t)(int)qf;
            if (y_out) y_out[(size_t)row * cols + c] = v[k];
        }
    }
}

// One warp per row (32-thread CTA), the row in registers (cols <= 32 x 4 x NV4, 16-byte
// aligned): the same LayerNorm and quantiser arithmetic as ln_quant_kernel with shuffle
// reductions instead of CTA-wide ones (decode rows are short).
template <int NV4>
__global__ void __launch_bounds__(32)
ln_quant_warp_kernel(int cols, const float* __restrict__ x, const float* __restrict__ gamma,
                     const float* __restrict__ beta, float eps, int32_t* __restrict__ q_out,
                     float* __restrict__ scale_out, float* __restrict__ y_out, __nv_bfloat16* __restrict__ y_hi,
                     __nv_bfloat16* __restrict__ y_lo) {
    griddep_wait();
    griddep_launch();
    const int row = blockIdx.x, lane = threadIdx.x;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * cols);
    const int c4 = cols >> 2;
    float4 v[NV4];
    float s = 0.f, ss = 0.f;
#pragma unroll
    for (int k = 0; k < NV4; ++k) {
        const int i = lane + 32 * k;
        v[k] = i < c4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
        ss = fmaf(v[k].x, v[k].x, ss);
        ss = fmaf(v[k].y, v[k].y, ss);
        ss = fmaf(v[k].z, v[k].z, ss);
        ss = fmaf(v[k].w, v[k].w, ss);
    }
    const float mean = warp_sum(s) / cols;
    const float var = warp_sum(ss) / cols - mean * mean;
    const float inv = rsqrtf(var + eps);
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < NV4; ++k) {
        const int i = lane + 32 * k;
        if (i < c4) {
            const float4 g = reinterpret_cast<const float4*>(gamma)[i];
            const float4 bb = reinterpret_cast<const float4*>(beta)[i];
            v[k].x = fmaf(g.x * (v[k].x - mean), inv, bb.x);
            v[k].y = fmaf(g.y * (v[k].y - mean), inv, bb.y);
            v[k].z = fmaf(g.z * (v[k].z - mean), inv, bb.z);
            v[k].w = fmaf(g.w * (v[k].w - mean), inv, bb.w);
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[k].x), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w))));
        }
    }
    if (!q_out) {  // plain LayerNorm (final ln_f feeding the vocab projection), fp32 and/or bf16 hi/lo
#pragma unroll
        for (int k = 0; k < NV4; ++k) {
            const int i = lane + 32 * k;
            if (i >= c4) continue;
            const float t[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
            if (y_out) reinterpret_cast<float4*>(y_out + (size_t)row * cols)[i] = v[k];
            if (y_hi) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const __nv_bfloat16 h = __float2bfloat16_rn(t[j]);
                    y_hi[(size_t)row * cols + 4 * i + j] = h;
                    y_lo[(size_t)row * cols + 4 * i + j] = __float2bfloat16_rn(t[j] - __bfloat162float(h));
                }
            }
        }
        return;
    }
    amax = warp_max(amax);
    // quantiser semantics of kernels/quantization/14_int8_gemm.cu:36-58
    const float scale = amax > 0.f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    const float invs = __fdiv_rn(1.0f, scale);
    if (lane == 0) scale_out[row] = scale;
    int32_t* qr = q_out + (size_t)row * c4;
#pragma unroll
    for (int k = 0; k < NV4; ++k) {
        const int i = lane + 32 * k;
        if (i >= c4) continue;
        const float t[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
        uint32_t packed = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float qf = fminf(fmaxf(rintf(__fmul_rn(t[j], invs)), -128.f), 127.f);
            packed |= (uint32_t)(uint8_t)(int8_t)(int)qf << (8 * j);
        }
        qr[i] = (int32_t)packed;
        if (y_out) reinterpret_cast<float4*>(y_out + (size_t)row * cols)[i] = v[k];
    }
}

// ------------------------------------------------------------------ QKV split + paged KV write
template <typename KV>
__device__ __forceinline__ KV to_kv(float v);
template <>
__device__ __forceinline__ float to_kv<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 to_kv<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename KV>
__global__ void qkv_scatter_kernel(int d, int H, int dh, int block_size, int nbps, const float* __restrict__ qkv,
                                   const int* __restrict__ pos, const int* __restrict__ block_table,
                                   float* __restrict__ q, KV* __restrict__ k_cache, KV* __restrict__ v_cache) {
    griddep_wait();
    griddep_launch();
    const int b = blockIdx.x;
    const int p = pos[b];
    const int phys = block_table[(size_t)b * nbps + p / block_size];
    const size_t slot = ((size_t)phys * block_size + p % block_size) * H * dh;  // token row base
    const float* src = qkv + (size_t)b * 3 * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        q[(size_t)b * d + i] = src[i];
        k_cache[slot + i] = to_kv<KV>(src[d + i]);
        v_cache[slot + i] = to_kv<KV>(src[2 * d + i]);
    }
}

// ------------------------------------------------------------------ vocab projection + argmax
// logits[b, v] = sum_k h[b,k] * wte[v,k] for a 64 x 64 (batch x vocab) tile per CTA, fp32 FMA
// in the reference's k order per output; then the tile's per-row maxima go to a 64-bit
// atomicMax whose key orders by value, then by lowest vocab index.
constexpr int VP_TB = 64, VP_TV = 64, VP_TK = 32, VP_THREADS = 256;

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

__global__ void __launch_bounds__(VP_THREADS)
vocab_argmax_kernel(int B, int V, int d, const float* __restrict__ h, const float* __restrict__ wte,
                    float* __restrict__ logits, unsigned long long* __restrict__ keys) {
    __shared__ float hs[VP_TK][VP_TB + 4];
    __shared__ float ws[VP_TK][VP_TV + 4];
    __shared__ unsigned long long best[VP_TB];
    griddep_wait();
    griddep_launch();
    const int v0 = blockIdx.x * VP_TV;
    const int b0 = blockIdx.y * VP_TB;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;  // 16 x 16 threads, 4 x 4 outputs each
    float acc[4][4] = {};
    for (int k0 = 0; k0 < d; k0 += VP_TK) {
        for (int i = threadIdx.x; i < VP_TK * VP_TB; i += VP_THREADS) {
            const int r = i / VP_TK, c = i % VP_TK;
            const int bb = b0 + r, kk = k0 + c;
            hs[c][r] = (bb < B && kk < d) ? h[(size_t)bb * d + kk] : 0.f;
            const int vv = v0 + r;
            ws[c][r] = (vv < V && kk < d) ? wte[(size_t)vv * d + kk] : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int c = 0; c < VP_TK; ++c) {
            float a[4], w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) { a[i] = hs[c][ty * 4 + i]; w[i] = ws[c][tx * 4 + i]; }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], w[j], acc[i][j]);
        }
        __syncthreads();
    }
    if (threadIdx.x < VP_TB) best[threadIdx.x] = 0ull;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int bb = b0 + ty * 4 + i;
        unsigned long long m = 0ull;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int vv = v0 + tx * 4 + j;
            if (bb < B && vv < V) {
                if (logits) logits[(size_t)bb * V + vv] = acc[i][j];
                const unsigned long long key = argmax_key(acc[i][j], vv);
                m = key > m ? key : m;
            }
        }
        if (bb < B) atomicMax(&best[ty * 4 + i], m);
    }
    __syncthreads();
    if (threadIdx.x < VP_TB && b0 + threadIdx.x < B) atomicMax(&keys[b0 + threadIdx.x], best[threadIdx.x]);
}

// next token = argmax (or the forced prompt token while the prompt lasts); advance positions
__global__ void advance_kernel(int B, const unsigned long long* __restrict__ keys, int* __restrict__ tokens,
                               int* __restrict__ pos, const int* __restrict__ forced, const int* __restrict__ forced_len,
                               int forced_stride, int* __restrict__ out_tokens, int out_stride, int max_pos) {
    griddep_wait();
    griddep_launch();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const int next = (int)(0xFFFFFFFFu - (uint32_t)(keys[b] & 0xFFFFFFFFull));
    const int p = min(pos[b] + 1, max_pos - 1);
    int tok = next;
    if (forced && p < forced_len[b]) tok = forced[(size_t)b * forced_stride + p];
    if (out_tokens && p < out_stride) out_tokens[(size_t)b * out_stride + p] = next;
    tokens[b] = tok;
    pos[b] = p;
}

// ------------------------------------------------------------------ launchers
int launch_embed(int B, int d, const int* tokens, const int* pos, const float* wte, const float* wpe, float* x,
                 int* ctx_lens, unsigned long long* keys, cudaStream_t st) {
    return launch_kernel(embed_kernel, dim3(B), dim3(256), 0, st, d, tokens, pos, wte, wpe, x, ctx_lens, keys) ==
                   cudaSuccess
               ? B2_OK
               : B2_ERR_CUDA;
}

int launch_ln_quant(int rows, int cols, const float* x, const float* gamma, const float* beta, float eps,
                    int32_t* q, float* scale, float* y, cudaStream_t st, void* y_hi, void* y_lo) {
    if (cols > LNQ_THREADS * LNQ_MAX_PER_THREAD || (cols & 3)) return B2_ERR_UNSUPPORTED;
    if (cols <= 4096 && ((uintptr_t)x & 15) == 0) {
        const int c4 = cols / 4;
        auto* hi = static_cast<__nv_bfloat16*>(y_hi);
        auto* lo = static_cast<__nv_bfloat16*>(y_lo);
        cudaError_t e;
        if (c4 <= 64)
            e = launch_kernel(ln_quant_warp_kernel<2>, dim3(rows), dim3(32), 0, st, cols, x, gamma, beta, eps, q, scale, y, hi, lo);
        else if (c4 <= 256)
            e = launch_kernel(ln_quant_warp_kernel<8>, dim3(rows), dim3(32), 0, st, cols, x, gamma, beta, eps, q, scale, y, hi, lo);
        else
            e = launch_kernel(ln_quant_warp_kernel<32>, dim3(rows), dim3(32), 0, st, cols, x, gamma, beta, eps, q, scale, y, hi, lo);
        return e == cudaSuccess ? B2_OK : B2_ERR_CUDA;
    }
    return launch_kernel(ln_quant_kernel, dim3(rows), dim3(LNQ_THREADS), 0, st, cols, x, gamma, beta, eps, q, scale,
                         y, static_cast<__nv_bfloat16*>(y_hi), static_cast<__nv_bfloat16*>(y_lo)) == cudaSuccess
               ? B2_OK
               : B2_ERR_CUDA;
}

int launch_qkv_scatter(int B, int d, int H, int dh, int block_size, int nbps, const float* qkv, const int* pos,
                       const int* block_table, float* q, void* k_cache, void* v_cache, int kv_dtype, cudaStream_t st) {
    cudaError_t e;
    if (kv_dtype == B2_KV_F32)
        e = launch_kernel(qkv_scatter_kernel<float>, dim3(B), dim3(256), 0, st, d, H, dh, block_size, nbps, qkv, pos,
                          block_table, q, static_cast<float*>(k_cache), static_cast<float*>(v_cache));
    else
        e = launch_kernel(qkv_scatter_kernel<__nv_bfloat16>, dim3(B), dim3(256), 0, st, d, H, dh, block_size, nbps,
                          qkv, pos, block_table, q, static_cast<__nv_bfloat16*>(k_cache),
                          static_cast<__nv_bfloat16*>(v_cache));
    return e == cudaSuccess ? B2_OK : B2_ERR_CUDA;
}

int launch_vocab_argmax(int B, int V, int d, const float* h, const float* wte, float* logits,
                        unsigned long long* keys, cudaStream_t st) {
    dim3 grid((V + VP_TV - 1) / VP_TV, (B + VP_TB - 1) / VP_TB);
    return launch_kernel(vocab_argmax_kernel, grid, dim3(VP_THREADS), 0, st, B, V, d, h, wte, logits, keys) ==
                   cudaSuccess
               ? B2_OK
               : B2_ERR_CUDA;
}

int launch_advance(int B, const unsigned long long* keys, int* tokens, int* pos, const int* forced,
                   const int* forced_len, int forced_stride, int* out_tokens, int out_stride, int max_pos,
                   cudaStream_t st) {
    return launch_kernel(advance_kernel, dim3((B + 127) / 128), dim3(128), 0, st, B, keys, tokens, pos, forced,
                         forced_len, forced_stride, out_tokens, out_stride, max_pos) == cudaSuccess
               ? B2_OK
               : B2_ERR_CUDA;
}

}  // namespace b2

// ------------------------------------------------------------------ tensor-parallel helpers
// A row-parallel linear needs the per-row scale of the FULL activation row, which is
// sharded across ranks: each rank takes its slice's absmax, an all-reduce(max) gives the
// global one, and every rank quantises its slice with it, so the int8 bytes equal those of
// the unsharded quantiser (kernels/quantization/14_int8_gemm.cu:22-58).
namespace b2 {

__global__ void rowmax_kernel(int cols, const float* __restrict__ x, float* __restrict__ amax_out) {
    griddep_wait();
    griddep_launch();
    __shared__ float red[8];
    const float* xr = x + (size_t)blockIdx.x * cols;
    float m = 0.f;
    for (int c = threadIdx.x; c < cols; c += 256) m = fmaxf(m, fabsf(xr[c]));
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
        m = fmaxf(m, red[0]);
        amax_out[blockIdx.x] = m;
    }
}

__global__ void quantize_scaled_kernel(int cols, const float* __restrict__ x, const float* __restrict__ amax,
                                       int32_t* __restrict__ q_out, float* __restrict__ scale_out) {
    griddep_wait();
    griddep_launch();
    const int row = blockIdx.x;
    const float a = amax[row];
    const float scale = a > 0.f ? __fdiv_rn(a, 127.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, scale);
    if (threadIdx.x == 0) scale_out[row] = scale;
    const float* xr = x + (size_t)row * cols;
    int8_t* qr = reinterpret_cast<int8_t*>(q_out) + (size_t)row * cols;
    for (int c = threadIdx.x; c < cols; c += 256)
        qr[c] = (int8_t)(int)fminf(fmaxf(rintf(__fmul_rn(xr[c], inv)), -128.f), 127.f);
}

// out[m, n] = epilogue(acc[m, n]) after the int32 all-reduce of a row-parallel linear.
template <int EPI>
__global__ void dequant_kernel(int M, int N, const int32_t* __restrict__ acc, const float* __restrict__ sA,
                               const float* __restrict__ sB, const float* __restrict__ bias,
                               const float* __restrict__ residual, float* __restrict__ out) {
    griddep_wait();
    griddep_launch();
    const size_t total = (size_t)M * N;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int m = (int)(i / N), n = (int)(i % N);
        const float rs = (EPI == B2_EPI_BIAS_RESIDUAL) ? residual[i] : 0.f;
        out[i] = epilogue<EPI>(acc[i], sA[m], sB[n], EPI != B2_EPI_PLAIN ? bias[n] : 0.f, rs);
    }
}

int launch_rowmax(int rows, int cols, const float* x, float* amax, cudaStream_t st) {
    return launch_kernel(rowmax_kernel, dim3(rows), dim3(256), 0, st, cols, x, amax) == cudaSuccess ? B2_OK
                                                                                                    : B2_ERR_CUDA;
}

int launch_quantize_scaled(int rows, int cols, const float* x, const float* amax, int32_t* q, float* scale,
                           cudaStream_t st) {
    return launch_kernel(quantize_scaled_kernel, dim3(rows), dim3(256), 0, st, cols, x, amax, q, scale) == cudaSuccess
               ? B2_OK
               : B2_ERR_CUDA;
}

int launch_dequant_residual(int M, int N, const int32_t* acc, const float* sA, const float* sB, const float* bias,
                            const float* residual, float* out, cudaStream_t st) {
    const int blocks = (int)std::min<size_t>(((size_t)M * N + 255) / 256, 1184);
    return launch_kernel(dequant_kernel<B2_EPI_BIAS_RESIDUAL>, dim3(blocks), dim3(256), 0, st, M, N, acc, sA, sB, bias,
                         residual, out) == cudaSuccess
               ? B2_OK
               : B2_ERR_CUDA;
}

}  // namespace b2
