// Causal attention of the engine's batched prefill (b2_engine_prefill).
//
// A prefill pass holds one row per prompt token (row r = position pos[r] of its sequence;
// rows of a sequence are consecutive, positions ascending). Row r attends to keys
// [0, pos[r]] of its own sequence through that sequence's block table, with the semantics
// of the decode attention (softmax(q.k * scale) . v, scale 1/sqrt(head_dim), fp32
// accumulation, fp32 or bf16 cache). Running every row as its own decode-attention unit
// costs one CTA per (row, head) of a few dozen tokens each; here a CTA takes PQ consecutive
// rows of one sequence (a work item from the host) for one head and streams the union of
// their key ranges once through shared memory, every K/V tile serving all PQ rows:
//   - K tiles are stored transposed ([head_dim][KT]) so that q.k runs with lanes over keys
//     (conflict-free), V tiles as rows for p.V with lanes over head_dim;
//   - each warp owns PQ/8 rows: per 32-key tile, 32 dot products per lane pass, a warp max
//     and sum for the online softmax (exp2 domain), and p broadcast by shuffles into p.V.
#include "common.cuh"
#include <cuda_bf16.h>

namespace b2 {

constexpr int PA_THREADS = 256;
constexpr int PA_WARPS = PA_THREADS / 32;
constexpr int PA_PQ = 16;   // query rows per CTA
constexpr int PA_KT = 32;   // keys per tile

template <typename KV>
__device__ __forceinline__ float kv_to_f32(KV v);
template <>
__device__ __forceinline__ float kv_to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float kv_to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// items[i] = (first row, row count <= PA_PQ) of one sequence; grid (heads, items).
template <int D, typename KV>
__global__ void __launch_bounds__(PA_THREADS)
prefill_attn_kernel(const int2* __restrict__ items, int H, const float* __restrict__ Q,
                    const KV* __restrict__ k_cache, const KV* __restrict__ v_cache, const int* __restrict__ block_table,
                    int nbps, int block_size, const int* __restrict__ pos, float scale_log2, float* __restrict__ O) {
    __shared__ float qs[PA_PQ][D];
    __shared__ float kt[D][PA_KT + 1];  // transposed K tile (+1: conflict-free column writes)
    __shared__ float vt[PA_KT][D];
    griddep_wait();
    griddep_launch();
    const int h = blockIdx.x;
    const int2 it = items[blockIdx.y];
    const int r0 = it.x, nq = it.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int* bt = block_table + (size_t)r0 * nbps;  // every row of the item shares its sequence's table
    for (int i = threadIdx.x; i < PA_PQ * D; i += PA_THREADS) {
        const int qi = i / D, c = i - qi * D;
        qs[qi][c] = qi < nq ? Q[((size_t)(r0 + qi) * H + h) * D + c] * scale_log2 : 0.f;
    }
    const int kend = pos[r0 + nq - 1] + 1;  // keys the last row sees (the widest range)
    constexpr int RPW = PA_PQ / PA_WARPS;   // rows per warp
    constexpr int VPL = D / 32;             // head_dim columns per lane in p.V
    float m[RPW], l[RPW], acc[RPW][VPL];
    int lim[RPW];
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
        const int qi = warp * RPW + j;
        m[j] = -INFINITY;
        l[j] = 0.f;
        lim[j] = qi < nq ? pos[r0 + qi] + 1 : 0;  // keys [0, lim) are visible to this row
#pragma unroll
        for (int c = 0; c < VPL; ++c) acc[j][c] = 0.f;
    }
    for (int t0 = 0; t0 < kend; t0 += PA_KT) {
        __syncthreads();  // the previous tile is consumed (and qs is written, first time)
        for (int i = threadIdx.x; i < PA_KT * D; i += PA_THREADS) {
            const int kk = i / D, c = i - kk * D;
            const int key = t0 + kk;
            float kf = 0.f, vf = 0.f;
            if (key < kend) {
                const int phys = bt[key / block_size];
                const size_t off = (((size_t)phys * block_size + key % block_size) * H + h) * D + c;
                kf = kv_to_f32<KV>(k_cache[off]);
                vf = kv_to_f32<KV>(v_cache[off]);
            }
            kt[c][kk] = kf;
            vt[kk][c] = vf;
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < RPW; ++j) {
            const int qi = warp * RPW + j;
            if (t0 >= lim[j]) continue;  // warp-uniform: this row's keys end before the tile
            // q.k for key t0 + lane
            float s = 0.f;
#pragma unroll 16
            for (int c = 0; c < D; ++c) s = fmaf(qs[qi][c], kt[c][lane], s);
            const bool valid = t0 + lane < lim[j];
            s = valid ? s : -INFINITY;
            const float tmax = warp_max(s);
            const float m_new = fmaxf(m[j], tmax);
            const float alpha = m[j] == -INFINITY ? 0.f : fast_exp2(m[j] - m_new);
            const float p = valid ? fast_exp2(s - m_new) : 0.f;
            l[j] = fmaf(l[j], alpha, warp_sum(p));
            m[j] = m_new;
#pragma unroll
            for (int c = 0; c < VPL; ++c) acc[j][c] *= alpha;
            const int kn = min(PA_KT, lim[j] - t0);
            for (int kk = 0; kk < kn; ++kk) {
                const float pk = __shfl_sync(0xffffffffu, p, kk);
#pragma unroll
                for (int c = 0; c < VPL; ++c) acc[j][c] = fmaf(pk, vt[kk][lane + 32 * c], acc[j][c]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
        const int qi = warp * RPW + j;
        if (qi >= nq) continue;
        float* o = O + ((size_t)(r0 + qi) * H + h) * D;
        const float inv = l[j] > 0.f ? 1.f / l[j] : 0.f;
#pragma unroll
        for (int c = 0; c < VPL; ++c) o[lane + 32 * c] = acc[j][c] * inv;
    }
}

// Rows of one launch: n_items work items (device array), H heads of head_dim D.
int launch_prefill_attention(const int2* items, int n_items, int H, int D, int kv_dtype, const float* q,
                             const void* k_cache, const void* v_cache, const int* block_table, int nbps,
                             int block_size, const int* pos, float* O, cudaStream_t st) {
    if (n_items <= 0) return B2_OK;
    const float scale_log2 = (1.0f / sqrtf((float)D)) * 1.4426950408889634f;
    dim3 grid(H, n_items);
    cudaError_t e = cudaErrorInvalidValue;
    const bool bf = kv_dtype == B2_KV_BF16;
    if (D == 64)
        e = bf ? launch_kernel(prefill_attn_kernel<64, __nv_bfloat16>, grid, dim3(PA_THREADS), 0, st, items, H, q,
                               static_cast<const __nv_bfloat16*>(k_cache), static_cast<const __nv_bfloat16*>(v_cache),
                               block_table, nbps, block_size, pos, scale_log2, O)
               : launch_kernel(prefill_attn_kernel<64, float>, grid, dim3(PA_THREADS), 0, st, items, H, q,
                               static_cast<const float*>(k_cache), static_cast<const float*>(v_cache), block_table, nbps,
                               block_size, pos, scale_log2, O);
    else if (D == 128)
        e = bf ? launch_kernel(prefill_attn_kernel<128, __nv_bfloat16>, grid, dim3(PA_THREADS), 0, st, items, H, q,
                               static_cast<const __nv_bfloat16*>(k_cache), static_cast<const __nv_bfloat16*>(v_cache),
                               block_table, nbps, block_size, pos, scale_log2, O)
               : launch_kernel(prefill_attn_kernel<128, float>, grid, dim3(PA_THREADS), 0, st, items, H, q,
                               static_cast<const float*>(k_cache), static_cast<const float*>(v_cache), block_table, nbps,
                               block_size, pos, scale_log2, O);
    return e == cudaSuccess ? B2_OK : B2_ERR_CUDA;
}

}  // namespace b2
