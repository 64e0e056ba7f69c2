// Fused collectives of the tensor-parallel decode step over NVLink peer memory.
//
// A row-parallel linear (attention out-projection, FC2) on rank r of `world` holds the
// activation columns [r*kl, (r+1)*kl) and the matching weight columns. Its exact
// single-GPU result needs (1) the per-row scale of the FULL activation row (max over ranks
// of each rank's row absmax) before int8 quantisation, and (2) the sum over ranks of the
// int32 partial products before the dequantisation epilogue. Instead of NCCL all-reduces
// around separate kernels, two kernels exchange through buffers every rank maps from every
// other rank (CUDA IPC), with epoch flags written by release stores and polled by acquire
// loads at system scope:
//
//   tp_quantize_kernel : per CTA one row: local |x| max -> stored into every rank's slot
//                        for this rank -> flag -> wait for every rank's flag -> global max ->
//                        scale, int8 quantisation of the local columns (bytes identical to
//                        the single-GPU quantiser's for those columns);
//   tp_reduce_kernel   : per CTA c: flag "my partials are final" -> wait for every rank's ->
//                        sum chunk (r, c) of the [B, d] int32 partials over all ranks (peer
//                        loads, exact) -> dequant + bias + residual -> the new residual chunk
//                        stored into every rank's x -> flag -> wait until every rank's chunk
//                        (r', c) has landed in this rank's x.
//
// Every wait is bounded (B2_WAIT_NS); a timeout sets B2_DEVERR_TIMEOUT and the kernel goes
// on, so a missing peer never hangs the GPU. Peers are reached with plain loads and stores
// (no multicast objects). Rank r owns chunk (r, c) of every call, so a rank only ever reads
// its own chunk of x as the residual while peers write the others.
#include "common.cuh"
#include "epilogue.cuh"
#include "tp_collectives.cuh"
#include <algorithm>

namespace b2 {

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Bounded wait until the flag holds epoch `ep` (or a later one).
__device__ __forceinline__ void wait_flag(const unsigned int* f, unsigned int ep, unsigned int* err) {
    if ((int)(ld_acquire_sys(f) - ep) >= 0) return;
    const uint64_t t0 = globaltimer();
    while ((int)(ld_acquire_sys(f) - ep) < 0) {
        if (globaltimer() - t0 > B2_WAIT_NS) {
            raise_error(err, B2_DEVERR_TIMEOUT);
            return;
        }
    }
}

__device__ __forceinline__ unsigned int* tp_flag(unsigned char* xchg, const TpLayout& L, int kind, int src, int cta) {
    return reinterpret_cast<unsigned int*>(xchg + L.flags) + (kind * TP_MAX_RANKS + src) * TP_MAX_CTAS + cta;
}
__device__ __forceinline__ unsigned int* tp_epoch(unsigned char* xchg, const TpLayout& L, int slot, int cta) {
    return reinterpret_cast<unsigned int*>(xchg + L.epochs) + slot * TP_MAX_CTAS + cta;
}

constexpr int TPQ_THREADS = 256;
constexpr int TPQ_CACHE = 8;  // float4 per thread kept in registers (rows up to 8192 columns)

// One CTA per row: |x| max of this rank's columns of the row -> every rank's slot -> flag ->
// wait for every rank -> global max -> scale and int8 quantisation of the local columns.
__global__ void __launch_bounds__(TPQ_THREADS)
tp_quantize_kernel(int kl, const float* __restrict__ x, int32_t* __restrict__ q_out, float* __restrict__ scale_out,
                   const TpPeers P) {
    __shared__ float red[TPQ_THREADS / 32];
    __shared__ unsigned int ep_s;
    griddep_wait();
    griddep_launch();
    const int row = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned char* mine = P.xchg[P.rank];
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * kl);
    const int n4 = kl / 4;
    float4 v[TPQ_CACHE];
    float m = 0.f;
#pragma unroll
    for (int k = 0; k < TPQ_CACHE; ++k) {
        const int i = threadIdx.x + k * TPQ_THREADS;
        v[k] = i < n4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v[k].x), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w))));
    }
    for (int i = threadIdx.x + TPQ_CACHE * TPQ_THREADS; i < n4; i += TPQ_THREADS) {
        const float4 t = xr[i];
        m = fmaxf(m, fmaxf(fmaxf(fabsf(t.x), fabsf(t.y)), fmaxf(fabsf(t.z), fabsf(t.w))));
    }
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    if (threadIdx.x == 0) ep_s = *tp_epoch(mine, P.L, 0, row) + 1;
    __syncthreads();
    const unsigned int ep = ep_s;
    if (threadIdx.x < P.world) {
        float a = red[0];
#pragma unroll
        for (int w = 1; w < TPQ_THREADS / 32; ++w) a = fmaxf(a, red[w]);
        // this rank's row maximum into slot [rank] of rank threadIdx.x, then its flag
        reinterpret_cast<float*>(P.xchg[threadIdx.x] + P.L.amax)[(size_t)P.rank * P.L.bmax + row] = a;
        __threadfence_system();
        st_release_sys(tp_flag(P.xchg[threadIdx.x], P.L, 0, P.rank, row), ep);
        wait_flag(tp_flag(mine, P.L, 0, threadIdx.x, row), ep, P.err);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const volatile float* slots = reinterpret_cast<const volatile float*>(mine + P.L.amax);
        float g = 0.f;
        for (int p = 0; p < P.world; ++p) g = fmaxf(g, slots[(size_t)p * P.L.bmax + row]);
        red[0] = g;
        *tp_epoch(mine, P.L, 0, row) = ep;
    }
    __syncthreads();
    // quantiser semantics of kernels/quantization/14_int8_gemm.cu:36-58 with the row's global absmax
    const float a = red[0];
    const float scale = a > 0.f ? __fdiv_rn(a, 127.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, scale);
    if (threadIdx.x == 0) scale_out[row] = scale;
    auto q4 = [&](float4 t) {
        const int b0 = (int)fminf(fmaxf(rintf(__fmul_rn(t.x, inv)), -128.f), 127.f);
        const int b1 = (int)fminf(fmaxf(rintf(__fmul_rn(t.y, inv)), -128.f), 127.f);
        const int b2 = (int)fminf(fmaxf(rintf(__fmul_rn(t.z, inv)), -128.f), 127.f);
        const int b3 = (int)fminf(fmaxf(rintf(__fmul_rn(t.w, inv)), -128.f), 127.f);
        return (int32_t)((b0 & 0xff) | ((b1 & 0xff) << 8) | ((b2 & 0xff) << 16) | ((uint32_t)(b3 & 0xff) << 24));
    };
    int32_t* qr = q_out + (size_t)row * n4;
#pragma unroll
    for (int k = 0; k < TPQ_CACHE; ++k) {
        const int i = threadIdx.x + k * TPQ_THREADS;
        if (i < n4) qr[i] = q4(v[k]);
    }
    for (int i = threadIdx.x + TPQ_CACHE * TPQ_THREADS; i < n4; i += TPQ_THREADS) qr[i] = q4(xr[i]);
}

constexpr int TPR_THREADS = 256;

__global__ void __launch_bounds__(TPR_THREADS)
tp_reduce_kernel(int B, int d, int chunk, const float* __restrict__ sA, const float* __restrict__ sB,
                 const float* __restrict__ bias, const TpPeers P) {
    __shared__ unsigned int ep_s;
    griddep_wait();  // this rank's GEMM partials are complete
    griddep_launch();
    const int c = blockIdx.x;
    unsigned char* mine = P.xchg[P.rank];
    if (threadIdx.x == 0) ep_s = *tp_epoch(mine, P.L, 1, c) + 1;
    __threadfence_system();
    __syncthreads();
    const unsigned int ep = ep_s;
    if (threadIdx.x < P.world) st_release_sys(tp_flag(P.xchg[threadIdx.x], P.L, 1, P.rank, c), ep);
    if (threadIdx.x < P.world) wait_flag(tp_flag(mine, P.L, 1, threadIdx.x, c), ep, P.err);
    __syncthreads();
    const size_t E = (size_t)B * d;
    const size_t base = ((size_t)P.rank * gridDim.x + c) * chunk;
    const size_t end = base + chunk < E ? base + chunk : E;
    const float* xl = P.x[P.rank];
    for (size_t i = base + 4 * (size_t)threadIdx.x; i < end; i += 4 * TPR_THREADS) {
        int4 v[TP_MAX_RANKS];
#pragma unroll
        for (int p = 0; p < TP_MAX_RANKS; ++p)
            if (p < P.world) v[p] = __ldcv(reinterpret_cast<const int4*>(P.acc[p] + i));
        int s[4] = {0, 0, 0, 0};
#pragma unroll
        for (int p = 0; p < TP_MAX_RANKS; ++p)
            if (p < P.world) { s[0] += v[p].x; s[1] += v[p].y; s[2] += v[p].z; s[3] += v[p].w; }
        const int m = (int)(i / d), n = (int)(i - (size_t)m * d);  // d % 4 == 0: one row
        const float4 r = *reinterpret_cast<const float4*>(xl + i);
        const float rs[4] = {r.x, r.y, r.z, r.w};
        float o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) o[q] = epilogue<B2_EPI_BIAS_RESIDUAL>(s[q], sA[m], sB[n + q], bias[n + q], rs[q]);
        const float4 ov = make_float4(o[0], o[1], o[2], o[3]);
#pragma unroll
        for (int p = 0; p < TP_MAX_RANKS; ++p)
            if (p < P.world) *reinterpret_cast<float4*>(P.x[p] + i) = ov;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < P.world) st_release_sys(tp_flag(P.xchg[threadIdx.x], P.L, 2, P.rank, c), ep);
    if (threadIdx.x < P.world) wait_flag(tp_flag(mine, P.L, 2, threadIdx.x, c), ep, P.err);
    if (threadIdx.x == 0) *tp_epoch(mine, P.L, 1, c) = ep;
}

int launch_tp_quantize(int B, int kl, const float* x, int32_t* q, float* scale, const TpPeers& P, cudaStream_t st) {
    if (B <= 0) return B2_OK;
    if (B > P.L.bmax || B > TP_MAX_CTAS || (kl & 3)) return B2_ERR_UNSUPPORTED;
    return launch_kernel(tp_quantize_kernel, dim3(B), dim3(TPQ_THREADS), 0, st, kl, x, q, scale, P) == cudaSuccess
               ? B2_OK
               : B2_ERR_CUDA;
}

int launch_tp_reduce(int B, int d, const float* sA, const float* sB, const float* bias, const TpPeers& P,
                     cudaStream_t st) {
    if (B <= 0) return B2_OK;
    if (d % 4) return B2_ERR_UNSUPPORTED;
    const size_t E = (size_t)B * d;
    const size_t per_rank = (E + P.world - 1) / P.world;
    const int ctas = (int)std::min<size_t>(TP_MAX_CTAS, std::max<size_t>(1, (per_rank + 1023) / 1024));
    const int chunk = (int)(((per_rank + ctas - 1) / ctas + 3) & ~(size_t)3);
    return launch_kernel(tp_reduce_kernel, dim3(ctas), dim3(TPR_THREADS), 0, st, B, d, chunk, sA, sB, bias, P) ==
                   cudaSuccess
               ? B2_OK
               : B2_ERR_CUDA;
}

}  // namespace b2

// ------------------------------------------------------------------ failure-path diagnostic
extern "C" size_t b2_tp_exchange_bytes(int rows) {
    return rows > 0 ? b2::TpLayout::make(rows).bytes : 0;
}

extern "C" int b2_tp_quantize_absent_peer(int rows, int cols, const float* x, int32_t* q_packed, float* scales,
                                          void* xchg_self, void* xchg_absent, b2_stream_t stream) {
    if (rows <= 0 || rows > b2::TP_MAX_CTAS || cols <= 0 || (cols & 3) || !x || !q_packed || !scales ||
        !xchg_self || !xchg_absent)
        return B2_ERR_INVALID;
    if (((uintptr_t)x | (uintptr_t)xchg_self | (uintptr_t)xchg_absent) & 15) return B2_ERR_INVALID;
    b2::TpPeers P;
    for (int r = 0; r < b2::TP_MAX_RANKS; ++r) {
        P.x[r] = nullptr;
        P.acc[r] = nullptr;
        P.xchg[r] = nullptr;
    }
    P.xchg[0] = static_cast<unsigned char*>(xchg_self);
    P.xchg[1] = static_cast<unsigned char*>(xchg_absent);
    P.L = b2::TpLayout::make(rows);
    P.rank = 0;
    P.world = 2;
    P.err = b2::device_error_ptr();
    if (!P.err) return B2_ERR_CUDA;
    return b2::launch_tp_quantize(rows, cols, x, q_packed, scales, P, static_cast<cudaStream_t>(stream));
}

