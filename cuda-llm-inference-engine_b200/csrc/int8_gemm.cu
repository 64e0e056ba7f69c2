// K14 on sm_100a: per-row symmetric INT8 quantiser and the INT8 GEMM on tcgen05.
//
// Quantiser semantics (reference kernels/quantization/14_int8_gemm.cu:10-60):
//   amax = max_k |x[r,k]|;  scale = amax > 0 ? amax / 127 : 1;  inv = 1 / scale (IEEE);
//   q = clamp(rint(x * inv), -128, 127) (round half to even);  packed little-endian 4 per int32.
// GEMM semantics (reference kernels/quantization/14_int8_gemm.cu:65-170):
//   acc = sum_k A[m,k] * B[n,k] (exact int32);  v = float(acc) * sA[m] * sB[n]
//   then  +bias[n]  /  +bias, GELU-tanh  /  +bias +residual[m,n].
// The reference's nvcc build contracts `v * sB + bias` into one fused multiply-add; the
// epilogue below spells the same operations out (fmaf) so results are bit-identical.
//
// B200 design of the GEMM (persistent, one CTA per SM, 128 x BN output tiles, 192 threads):
//   warp 0  : TMA producer — 2-D tensor-map loads of 128 x 128-byte A and BN x 128-byte B
//             tiles in the 128-byte swizzle into a STAGES-deep ring (mbarrier full/empty);
//   warp 1  : allocates BN TMEM columns and issues tcgen05.mma.cta_group::1.kind::i8
//             (M=128, N=BN, K=32 per instruction, int32 accumulators in TMEM), releasing
//             ring slots with tcgen05.commit;
//   warps 2-5: epilogue — tcgen05.ld of the accumulator (one TMEM lane quadrant per warp,
//             thread = output row), dequantise + bias / GELU / residual in registers, store.
//   Two TMEM accumulators (2 x BN columns) let the epilogue of tile j overlap the MMAs of
//   tile j+1; tiles are visited in groups of 8 row-tiles so concurrently running CTAs
//   share A and B tiles in L2.
#include "common.cuh"
#include "epilogue.cuh"
#include "rowops.cuh"
#include "engine_kernels.cuh"
#include <cuda_bf16.h>
#include <algorithm>
#include <cmath>
#include <mutex>

namespace b2 {

// ------------------------------------------------------------------ quantiser
constexpr int QZ_THREADS = 256;

__global__ void __launch_bounds__(QZ_THREADS)
quantize_rows_kernel(int cols, const float* __restrict__ in, int32_t* __restrict__ out,
                     float* __restrict__ scales) {
    griddep_wait();
    griddep_launch();
    const int row = blockIdx.x;
    const float* x = in + (size_t)row * cols;
    const int c4 = cols >> 2;
    const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    float amax = 0.f;
    if (vec) {
        const float4* x4 = reinterpret_cast<const float4*>(x);
        for (int i = threadIdx.x; i < c4; i += QZ_THREADS) {
            float4 v = x4[i];
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    } else {
        for (int i = threadIdx.x; i < cols; i += QZ_THREADS) amax = fmaxf(amax, fabsf(x[i]));
    }
    __shared__ float red[QZ_THREADS / 32];
    amax = warp_max(amax);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int w = 1; w < QZ_THREADS / 32; ++w) amax = fmaxf(amax, red[w]);
    const float scale = amax > 0.f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, scale);
    if (threadIdx.x == 0) scales[row] = scale;
    int32_t* o = out + (size_t)row * c4;
    for (int i = threadIdx.x; i < c4; i += QZ_THREADS) {
        float v[4];
        if (vec) {
            float4 t = reinterpret_cast<const float4*>(x)[i];
            v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        } else {
            v[0] = x[4 * i]; v[1] = x[4 * i + 1]; v[2] = x[4 * i + 2]; v[3] = x[4 * i + 3];
        }
        uint32_t packed = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float q = fminf(fmaxf(rintf(__fmul_rn(v[j], inv)), -128.f), 127.f);
            packed |= (uint32_t)(uint8_t)(int8_t)(int)q << (8 * j);
        }
        o[i] = (int32_t)packed;
    }
}

// Rows of at most 32 x 4 x NV4 columns (16-byte aligned): one warp per row in a 32-thread
// CTA, the row held in registers, shuffle reductions only (decode rows are short: a CTA-wide
// reduction costs more than the row's bytes).
template <int NV4>
__global__ void __launch_bounds__(32)
quantize_rows_warp_kernel(int cols, const float* __restrict__ in, int32_t* __restrict__ out,
                          float* __restrict__ scales) {
    griddep_wait();
    griddep_launch();
    const size_t row = blockIdx.x;
    quant_row_warp<NV4>(in + row * cols, cols, out + row * (cols >> 2), scales + row, threadIdx.x);
}

int quantize_launch(int rows, int cols, const float* in, int32_t* out, float* scales, cudaStream_t st) {
    if (rows < 0 || cols < 0 || (cols & 3)) return B2_ERR_INVALID;
    if (rows == 0) return B2_OK;
    if (!in || !out || !scales) return B2_ERR_INVALID;
    cudaError_t e;
    if (((uintptr_t)in & 15) == 0 && cols <= 4096) {
        const int c4 = (cols + 3) / 4;
        if (c4 <= 64)
            e = launch_kernel(quantize_rows_warp_kernel<2>, dim3(rows), dim3(32), 0, st, cols, in, out, scales);
        else if (c4 <= 256)
            e = launch_kernel(quantize_rows_warp_kernel<8>, dim3(rows), dim3(32), 0, st, cols, in, out, scales);
        else
            e = launch_kernel(quantize_rows_warp_kernel<32>, dim3(rows), dim3(32), 0, st, cols, in, out, scales);
    } else {
        e = launch_kernel(quantize_rows_kernel, dim3(rows), dim3(QZ_THREADS), 0, st, cols, in, out, scales);
    }
    return e == cudaSuccess ? B2_OK : B2_ERR_CUDA;
}

// ------------------------------------------------------------------ tcgen05 GEMM
constexpr int GM_BM = 128;
constexpr int GM_BK = 128;  // bytes of K per stage (one 128-byte swizzle atom row)
constexpr int GM_THREADS = 192;

// Destination of a fused QKV epilogue (decode engine): output column n of row b belongs to
// q (n < d), K (d <= n < 2d) or V; q goes to q[b, n], K/V to the paged cache row of token
// pos[b] of sequence b: cache[((phys * bs + pos % bs) * d + n % d)] with
// phys = block_table[b * nbps + pos / bs] (layout [P, bs, H, d_head], d = H * d_head).
struct QkvScatter {
    float* q = nullptr;
    void* k = nullptr;
    void* v = nullptr;
    const int* pos = nullptr;
    const int* block_table = nullptr;
    int d = 0, bs = 0, nbps = 0, bf16 = 0;
};

struct GemmParams {
    int M, N, K;
    const float* scale_A;
    const float* scale_B;
    const float* bias;
    const float* residual;
    void* C;  // float* or int32_t*
    unsigned int* err;
    // split-K (decode-size GEMMs): k_splits ranges of kb_per_split k-blocks per tile; int32
    // partials in ws [k_splits][M][N]; counters [tiles] arrival tickets, zero at rest
    int k_splits, kb_per_split;
    int32_t* ws;
    unsigned int* counters;
    // rows of A each stage loads (box height of A's tensor map): 128, or M rounded up to 8
    // when the output has a single 128-row tile (rows past it hold stale data whose
    // accumulator rows the epilogue never stores)
    int a_rows;
    QkvScatter sc;  // sc.q != nullptr: the engine's fused QKV split + paged KV write
    // the weights (B) are constant, so their first ring stages may be requested before the
    // kernel waits on the previous grid (the decode engine); otherwise every global read
    // follows the wait, which makes programmatic dependent launch safe for any producer
    int b_early;
    // the k_splits CTAs of a tile form a thread-block cluster. 1: ranks 1.. hand their int32
    // partials to rank 0's shared memory (GemmCfg::RED_BYTES), which sums them and stores
    // the tile; 2 (reduce-scatter): rank r owns the tile's columns [r S, (r+1) S),
    // S = BN / k_splits, receives every partner's partial of them through exchange rows in
    // ws and stores them
    int cluster_k;
};

template <int BN>
struct GemmCfg {
    static constexpr int A_BYTES = GM_BM * GM_BK;
    static constexpr int B_BYTES = BN * GM_BK;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    // cluster partials: 32-column tiles gather up to 3 partners' 128 x 32 int32 partials in
    // rank 0 (the reduce-scatter of 128-column tiles exchanges through global memory)
    static constexpr int RED_MAX = 3;
    static constexpr int RED_BYTES = BN == 32 ? RED_MAX * GM_BM * BN * 4 : 0;
    static constexpr int STAGES = std::min(8, (196 * 1024 - RED_BYTES) / STAGE);
    static constexpr int OFF_RED = STAGES * STAGE;
    static constexpr int OFF_BAR = OFF_RED + RED_BYTES;
    // full[S], empty[S], acc_full[2], acc_empty[2], drain, red (cluster partials landed)
    static constexpr int NBAR = 2 * STAGES + 6;
    static constexpr int OFF_COL = OFF_BAR + NBAR * 8 + 16;      // f32 [2][BN]: scale_B, bias of the tile
    static constexpr int SMEM = OFF_COL + 2 * BN * 4 + 1024;     // + 1 KB for alignment
    static constexpr uint32_t ACC_COLS = BN < 32 ? 32 : BN;      // one accumulator
    static constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;          // double-buffered
};

constexpr int GM_GROUP_M = 8;  // tile rasterisation: 8 row-tiles share each sweep over N

// Tile index -> (m-tile, n-tile), grouped so CTAs running together reuse A and B in L2.
__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int& mt, int& nt) {
    const int per_group = GM_GROUP_M * n_tiles;
    const int group = t / per_group;
    const int first_m = group * GM_GROUP_M;
    const int gsize = min(m_tiles - first_m, GM_GROUP_M);
    const int r = t - group * per_group;
    mt = first_m + r % gsize;
    nt = r / gsize;
}

// Dequantise + epilogue for 16 consecutive columns [n, n+16) of one row, then store.
// sBs / bis point at the tile's column scales / biases staged in shared memory (index
// relative to n); rs holds the residual values when EPI needs them.
template <int EPI, bool S32>
__device__ __forceinline__ void store16(const uint32_t (&r)[16], int row, int n, float sa, const float* sBs,
                                        const float* bis, const float (&rs)[16], const GemmParams& p,
                                        long long sc_row = -1) {
    if constexpr (S32) {
        int32_t* Crow = static_cast<int32_t*>(p.C) + (size_t)row * p.N;
        if (n + 16 <= p.N && (p.N & 3) == 0) {
#pragma unroll
            for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<int4*>(Crow + n + j) = make_int4(r[j], r[j + 1], r[j + 2], r[j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (n + j < p.N) Crow[n + j] = (int32_t)r[j];
        }
    } else {
        float* Crow = static_cast<float*>(p.C) + (size_t)row * p.N;
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
            v[j] = epilogue<EPI>((int32_t)r[j], sa, sBs[j], EPI != B2_EPI_PLAIN ? bis[j] : 0.f, rs[j]);
        if (p.sc.q) {  // fused QKV split: 16 columns never straddle q/K/V (d % 16 == 0)
            const int part = n / p.sc.d, i = n - part * p.sc.d;
            if (part == 0) {
                float* dst = p.sc.q + (size_t)row * p.sc.d + i;
#pragma unroll
                for (int j = 0; j < 16; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
                const size_t off = (size_t)sc_row + i;
                void* cache = part == 1 ? p.sc.k : p.sc.v;
                if (p.sc.bf16) {
                    uint32_t w[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        w[j] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * j])) |
                               ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v[2 * j + 1])) << 16);
                    uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(cache) + off);
                    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
                } else {
                    float* dst = static_cast<float*>(cache) + off;
#pragma unroll
                    for (int j = 0; j < 16; j += 4)
                        *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                }
            }
            return;
        }
        if (n + 16 <= p.N && (p.N & 3) == 0) {
#pragma unroll
            for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<float4*>(Crow + n + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (n + j < p.N) Crow[n + j] = v[j];
        }
    }
}

// Residual values [n, n+16) of one row (zeros past N).
__device__ __forceinline__ void load_res16(const GemmParams& p, int row, int n, float (&rs)[16]) {
    const float* R = p.residual + (size_t)row * p.N + n;
    if (n + 16 <= p.N && (p.N & 3) == 0) {
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
            const float4 t = __ldg(reinterpret_cast<const float4*>(R + j));
            rs[j] = t.x; rs[j + 1] = t.y; rs[j + 2] = t.z; rs[j + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) rs[j] = (n + j < p.N) ? R[j] : 0.f;
    }
}

// Persistent: CTA c processes tiles c, c + gridDim.x, ... The TMA ring runs continuously
// across tiles, and two TMEM accumulators let the epilogue of one tile overlap the MMAs
// of the next.
template <int BN, int EPI, bool S32>
__global__ void __launch_bounds__(GM_THREADS, 1)
int8_gemm_tc_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                    const GemmParams p) {
    using C = GemmCfg<BN>;
    extern __shared__ unsigned char smem_raw[];
    // 1024-byte alignment for the 128-byte swizzle atoms
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + C::OFF_BAR;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (C::STAGES + s); };
    auto accf_bar = [&](int a) { return bar0 + 8u * (2 * C::STAGES + a); };
    auto acce_bar = [&](int a) { return bar0 + 8u * (2 * C::STAGES + 2 + a); };
    const uint32_t drain_bar = bar0 + 8u * (2 * C::STAGES + 4);  // the MMA issuer's drain after an abort
    const uint32_t red_bar = bar0 + 8u * (2 * C::STAGES + 5);    // cluster partials landed (rank 0)
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + C::OFF_BAR + C::NBAR * 8);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nk = (p.K + GM_BK - 1) / GM_BK;
    const int m_tiles = (p.M + GM_BM - 1) / GM_BM;
    const int n_tiles = (p.N + BN - 1) / BN;
    const int num_tiles = m_tiles * n_tiles;
    const int num_units = num_tiles * p.k_splits;  // work unit = (tile, k range)

    if (threadIdx.x == 0) {
        prefetch_tensormap(&mapA);
        prefetch_tensormap(&mapB);
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(accf_bar(a), 1);   // tcgen05.commit of the tile's last MMA
            mbar_init(acce_bar(a), 4);   // one arrival per epilogue warp
        }
        mbar_init(drain_bar, 1);
        mbar_init(red_bar, p.cluster_k ? (p.k_splits - 1) * 128 : 1);  // every epilogue thread of every partner
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(const_cast<uint32_t*>(tmem_slot)), C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    if (p.cluster_k) cluster_sync();  // rank 0's barrier is initialised before partners arrive on it
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------------------------------------------------------- TMA producer
            const uint64_t pol = policy_evict_last();
            // The weights (B) never depend on the previous kernel: the first ring stages'
            // B tiles are requested before waiting on it (programmatic dependent launch),
            // the activation (A) tiles after.
            int npre = 0;
            if (p.b_early && (int)blockIdx.x < num_units) {
                const int w = blockIdx.x;
                const int kb0 = (w % p.k_splits) * p.kb_per_split;
                const int kb1 = min(nk, kb0 + p.kb_per_split);
                int mt, nt;
                tile_coords(w / p.k_splits, m_tiles, n_tiles, mt, nt);
                npre = min(C::STAGES, kb1 - kb0);
                for (int i = 0; i < npre; ++i) {
                    const uint32_t b_s = sbase + i * C::STAGE + C::A_BYTES;
                    mbar_arrive_expect_tx(full_bar(i), p.a_rows * GM_BK + C::B_BYTES);
                    tma_load_2d(b_s, &mapB, (kb0 + i) * GM_BK, nt * BN, full_bar(i), pol);
                }
            }
            griddep_wait();
            griddep_launch();
            int it = 0;  // k-block counter across all tiles of this CTA
            for (int w = blockIdx.x; w < num_units && !*abort_flag; w += gridDim.x) {
                const int t = w / p.k_splits;
                const int kb0 = (w % p.k_splits) * p.kb_per_split;
                const int kb1 = min(nk, kb0 + p.kb_per_split);
                int mt, nt;
                tile_coords(t, m_tiles, n_tiles, mt, nt);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % C::STAGES;
                    const uint32_t a_s = sbase + s * C::STAGE;
                    const uint32_t b_s = a_s + C::A_BYTES;
                    if (it < npre) {  // B already requested
                        tma_load_2d(a_s, &mapA, kb * GM_BK, mt * GM_BM, full_bar(s), pol);
                        continue;
                    }
                    if (it >= C::STAGES) {
                        if (*abort_flag || !mbar_wait(empty_bar(s), ((it / C::STAGES) - 1) & 1, p.err)) {
                            *abort_flag = 1;
                            break;
                        }
                    }
                    mbar_arrive_expect_tx(full_bar(s), p.a_rows * GM_BK + C::B_BYTES);
                    tma_load_2d(a_s, &mapA, kb * GM_BK, mt * GM_BM, full_bar(s), pol);
                    tma_load_2d(b_s, &mapB, kb * GM_BK, nt * BN, full_bar(s), pol);
                }
            }
            // drain: the last fill of every stage this thread requested has landed before the
            // CTA can exit, also when a consumer gave up waiting (a prefetched fill whose A
            // tile was never requested cannot complete; its bounded wait covers the B tile)
            for (int j = max(0, it - C::STAGES); j < max(it, npre); ++j)
                mbar_wait_drain(full_bar(j % C::STAGES), (j / C::STAGES) & 1);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------------------------------------------------------- MMA issuer
            constexpr uint32_t idesc = idesc_i8(GM_BM, BN);
            int it = 0, j = 0;  // k-block counter, local tile counter
            for (int w = blockIdx.x; w < num_units && !*abort_flag; w += gridDim.x, ++j) {
                const int kb0 = (w % p.k_splits) * p.kb_per_split;
                const int kb1 = min(nk, kb0 + p.kb_per_split);
                const int a = j & 1, u = j >> 1;
                if (u >= 1 && !mbar_wait(acce_bar(a), (u - 1) & 1, p.err)) { *abort_flag = 1; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem + a * C::ACC_COLS;
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % C::STAGES;
                    if (*abort_flag || !mbar_wait(full_bar(s), (it / C::STAGES) & 1, p.err)) {
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_s = sbase + s * C::STAGE;
                    const uint32_t b_s = a_s + C::A_BYTES;
                    const uint64_t da = smem_desc_sw128(a_s);
                    const uint64_t db = smem_desc_sw128(b_s);
#pragma unroll
                    for (int k = 0; k < GM_BK / 32; ++k) {
                        // advance 32 bytes of K inside the swizzle atom: +2 in the 16-byte address field
                        mma_i8(d_tmem, da + 2 * k, db + 2 * k, idesc, ((kb - kb0) | k) != 0 ? 1u : 0u);
                    }
                    mma_commit(empty_bar(s));  // ring slot free once these MMAs have read it
                }
                mma_commit(accf_bar(a));  // accumulator a complete
            }
            if (*abort_flag) {  // drain: every MMA issued has finished before TMEM is freed
                mma_commit(drain_bar);
                mbar_wait_drain(drain_bar, 0);
            }
        }
        __syncwarp();
    } else {
        // -------------------------------------------------------------------- epilogue
        const int quad = warp & 3;  // TMEM lane quadrant this warp may access
        const int et = threadIdx.x - 64;  // 0..127 across the epilogue warps
        griddep_wait();                   // scale_A / residual may come from the previous kernel
        float* sB_s = reinterpret_cast<float*>(smem + C::OFF_COL);
        float* bias_s = sB_s + BN;
        int j = 0;
        for (int w = blockIdx.x; w < num_units; w += gridDim.x, ++j) {
            const int t = w / p.k_splits;
            const int ksi = w % p.k_splits;
            const int a = j & 1, u = j >> 1;
            int mt, nt;
            tile_coords(t, m_tiles, n_tiles, mt, nt);
            // stage this tile's column scales and biases while the MMAs run
            if constexpr (!S32) {
                for (int c = et; c < BN; c += 128) {
                    const int n = nt * BN + c;
                    sB_s[c] = n < p.N ? __ldg(p.scale_B + n) : 0.f;
                    if (EPI != B2_EPI_PLAIN) bias_s[c] = n < p.N ? __ldg(p.bias + n) : 0.f;
                }
            }
            // fused QKV split: this row's paged-cache row offset, looked up while the MMAs run
            long long sc_row = 0;
            if (p.sc.q) {
                const int r = mt * GM_BM + quad * 32 + lane;
                if (r < p.M) {
                    const int pos = p.sc.pos[r];
                    const int phys = p.sc.block_table[(size_t)r * p.sc.nbps + pos / p.sc.bs];
                    sc_row = ((long long)phys * p.sc.bs + pos % p.sc.bs) * p.sc.d;
                }
            }
            named_barrier(2, 128);
            // after a timed-out wait the warps keep taking the named barriers but do no work
            const bool ok = !*abort_flag && mbar_wait(accf_bar(a), u & 1, p.err);
            if (!ok) *abort_flag = 1;
            tc_fence_after();
            const int row = mt * GM_BM + quad * 32 + lane;
            const bool row_ok = ok && row < p.M;
            const float sa = (!S32 && row_ok) ? __ldg(p.scale_A + row) : 0.f;
            const uint32_t tbase = tmem + a * C::ACC_COLS + ((uint32_t)(quad * 32) << 16);
            // final dequantise/epilogue/store of columns [n, n+32) from accumulators r0, r1
            auto finish32 = [&](const uint32_t (&r0)[16], const uint32_t (&r1)[16], int c) {
                const int n = nt * BN + c * 16;
                float rs0[16], rs1[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) { rs0[i] = 0.f; rs1[i] = 0.f; }
                if constexpr (EPI == B2_EPI_BIAS_RESIDUAL && !S32) {
                    if (row_ok && n < p.N) load_res16(p, row, n, rs0);
                    if (row_ok && n + 16 < p.N) load_res16(p, row, n + 16, rs1);
                }
                if (row_ok && n < p.N) store16<EPI, S32>(r0, row, n, sa, sB_s + c * 16, bias_s + c * 16, rs0, p, sc_row);
                if (row_ok && n + 16 < p.N)
                    store16<EPI, S32>(r1, row, n + 16, sa, sB_s + c * 16 + 16, bias_s + c * 16 + 16, rs1, p, sc_row);
            };
            if (p.k_splits == 1) {
#pragma unroll 1
                for (int c = 0; c < BN / 16; c += 2) {
                    uint32_t r0[16], r1[16];
                    tmem_ld16(tbase + (uint32_t)(c * 16), r0);
                    tmem_ld16(tbase + (uint32_t)(c * 16 + 16), r1);
                    tmem_ld_wait();
                    finish32(r0, r1, c);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(acce_bar(a));  // accumulator a may be overwritten
            } else if (p.cluster_k == 2) {
                // cluster reduce-scatter: rank ksi owns the tile's columns [ksi S, ksi S + S).
                // It writes every other slice of its int32 partial to the owner's exchange
                // rows in global memory (L2: distributed shared memory moves only ~30-40 GB/s
                // per SM in an all-to-all), arrives on the owner's barrier with release at
                // cluster scope, waits (acquire) for its own partners, adds the slices they
                // wrote to its own (exact) and runs the epilogue on its columns. Exchange rows
                // are laid out [tile][owner][slot][granule][row] (16-byte granules), so a warp's
                // 32 rows of one granule are 512 contiguous bytes.
                const int S = BN / p.k_splits;  // 16, 32 or 64 columns
                const int G4 = S / 4;           // 16-byte granules per slice row
                const int lrow = quad * 32 + lane;
                const size_t slice_i4 = (size_t)G4 * GM_BM;  // int4 per (owner, slot) slice
                int4* xt = reinterpret_cast<int4*>(p.ws) + (size_t)t * p.k_splits * (p.k_splits - 1) * slice_i4;
#pragma unroll 1
                for (int pr = 1; pr < p.k_splits; ++pr) {
                    const int dst = (ksi + pr) % p.k_splits;  // staggered: partners fill different owners first
                    const int slot = ksi < dst ? ksi : ksi - 1;
                    int4* xs = xt + ((size_t)dst * (p.k_splits - 1) + slot) * slice_i4 + lrow;
#pragma unroll 1
                    for (int c = 0; c < S / 16; ++c) {
                        uint32_t r[16];
                        tmem_ld16(tbase + (uint32_t)(dst * S + c * 16), r);
                        tmem_ld_wait();
                        if (row_ok)
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                __stcg(xs + (size_t)(c * 4 + q) * GM_BM,
                                       make_int4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]));
                    }
                }
                // one release for all the stores above (a releasing arrive per owner would wait
                // for its stores each time); then lane j arrives for the whole warp on owner
                // ksi + 1 + j, so the remote arrivals go out in one instruction
                asm volatile("fence.acq_rel.cluster;" ::: "memory");
                __syncwarp();
                if (lane < p.k_splits - 1)
                    mbar_arrive_cluster_count(mapa_shared(red_bar, (uint32_t)((ksi + 1 + lane) % p.k_splits)), 32u);
                const bool got = ok && mbar_wait_cluster(red_bar, 0, p.err);
                if (!got) *abort_flag = 1;
                const int4* xo = xt + (size_t)ksi * (p.k_splits - 1) * slice_i4 + lrow;
#pragma unroll 1
                for (int c = 0; c < S / 16; ++c) {
                    uint32_t r[16];
                    tmem_ld16(tbase + (uint32_t)(ksi * S + c * 16), r);
                    tmem_ld_wait();
                    if (got && row_ok) {
                        // the partners' slices in batches of 4, every load of a batch in flight
                        const int ns = p.k_splits - 1;
                        for (int sl0 = 0; sl0 < ns; sl0 += 4) {
                            int4 v[4][4];
#pragma unroll
                            for (int j = 0; j < 4; ++j)
#pragma unroll
                                for (int q = 0; q < 4; ++q)
                                    v[j][q] = sl0 + j < ns ? __ldcg(xo + (sl0 + j) * slice_i4 + (size_t)(c * 4 + q) * GM_BM)
                                                           : make_int4(0, 0, 0, 0);
#pragma unroll
                            for (int j = 0; j < 4; ++j)
#pragma unroll
                                for (int q = 0; q < 4; ++q) {
                                    r[4 * q] = (uint32_t)((int32_t)r[4 * q] + v[j][q].x);
                                    r[4 * q + 1] = (uint32_t)((int32_t)r[4 * q + 1] + v[j][q].y);
                                    r[4 * q + 2] = (uint32_t)((int32_t)r[4 * q + 2] + v[j][q].z);
                                    r[4 * q + 3] = (uint32_t)((int32_t)r[4 * q + 3] + v[j][q].w);
                                }
                        }
                        const int cc = (ksi * S) / 16 + c;  // 16-column chunk of the tile
                        const int n = nt * BN + cc * 16;
                        float rs[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) rs[i] = 0.f;
                        if constexpr (EPI == B2_EPI_BIAS_RESIDUAL && !S32) {
                            if (n < p.N) load_res16(p, row, n, rs);
                        }
                        if (n < p.N) store16<EPI, S32>(r, row, n, sa, sB_s + cc * 16, bias_s + cc * 16, rs, p, sc_row);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(acce_bar(a));
            } else if (p.cluster_k) {
                // cluster split-K: partners push their int32 partials (valid rows only) into
                // rank 0's shared memory and arrive on its barrier; rank 0 adds them (exact)
                // to its own accumulator and runs the epilogue
                const int lrow = quad * 32 + lane;  // row within the tile
                if (ksi != 0) {
                    const uint32_t red_l = smem_u32(smem + C::OFF_RED) +
                                           (uint32_t)(((ksi - 1) * GM_BM + lrow) * BN * 4);
                    const uint32_t red_r = mapa_shared(red_l, 0);
#pragma unroll 1
                    for (int c = 0; c < BN / 16; ++c) {
                        uint32_t r[16];
                        tmem_ld16(tbase + (uint32_t)(c * 16), r);
                        tmem_ld_wait();
                        if (row_ok)
#pragma unroll
                            for (int q = 0; q < 16; q += 4)
                                st_cluster_v4(red_r + (uint32_t)((c * 16 + q) * 4),
                                              make_uint4(r[q], r[q + 1], r[q + 2], r[q + 3]));
                    }
                    tc_fence_before();
                    mbar_arrive_cluster(mapa_shared(red_bar, 0));  // release: the stores above
                    __syncwarp();
                    if (lane == 0) mbar_arrive(acce_bar(a));
                } else {
                    const bool got = ok && mbar_wait_cluster(red_bar, 0, p.err);
                    if (!got) *abort_flag = 1;
                    const int32_t* red = reinterpret_cast<const int32_t*>(smem + C::OFF_RED) + lrow * BN;
#pragma unroll 1
                    for (int c = 0; c < BN / 16; c += 2) {
                        uint32_t r0[16], r1[16];
                        tmem_ld16(tbase + (uint32_t)(c * 16), r0);
                        tmem_ld16(tbase + (uint32_t)(c * 16 + 16), r1);
                        tmem_ld_wait();
                        if (got && row_ok) {
                            for (int ks = 1; ks < p.k_splits; ++ks) {
                                const int32_t* src = red + (ks - 1) * GM_BM * BN + c * 16;
#pragma unroll
                                for (int q = 0; q < 16; ++q) {
                                    r0[q] = (uint32_t)((int32_t)r0[q] + src[q]);
                                    r1[q] = (uint32_t)((int32_t)r1[q] + src[16 + q]);
                                }
                            }
                            finish32(r0, r1, c);
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(acce_bar(a));
                }
            } else {
                // split-K: park this k range's int32 partial, then the last of the k_splits
                // arrivals for these 32 rows sums the partials (exact) and runs the epilogue
                int32_t* part = p.ws + (size_t)ksi * p.M * p.N;
#pragma unroll 1
                for (int c = 0; c < BN / 16; ++c) {
                    uint32_t r[16];
                    tmem_ld16(tbase + (uint32_t)(c * 16), r);
                    tmem_ld_wait();
                    const int n = nt * BN + c * 16;
                    if (row_ok && n < p.N) {
                        int32_t* dst = part + (size_t)row * p.N + n;
                        if (n + 16 <= p.N && (p.N & 3) == 0) {
#pragma unroll
                            for (int q = 0; q < 16; q += 4)
                                __stcg(reinterpret_cast<int4*>(dst + q), make_int4(r[q], r[q + 1], r[q + 2], r[q + 3]));
                        } else {
#pragma unroll
                            for (int q = 0; q < 16; ++q)
                                if (n + q < p.N) __stcg(dst + q, (int32_t)r[q]);
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(acce_bar(a));  // TMEM read out: accumulator a is free
                __threadfence();
                named_barrier(2, 128);  // all four warps have parked their rows
                volatile uint32_t* tk = tmem_slot + 2;
                unsigned int* ctr = p.counters + t;
                if (et == 0) *tk = atomicAdd(ctr, 1u);
                named_barrier(2, 128);
                if (*tk == (unsigned)(p.k_splits - 1)) {
                    // last k range of this tile: the 128 epilogue threads sum the partials with
                    // coalesced 16-byte loads (k ranges unrolled 4 deep) and run the epilogue
                    __threadfence();
                    const int r0 = mt * GM_BM;
                    const int rows = min(GM_BM, p.M - r0);
                    constexpr int C4 = BN / 4;
                    const bool vec = (p.N & 3) == 0;
                    for (int u = et; u < rows * C4; u += 128) {
                        const int row_i = r0 + u / C4;
                        const int cl = (u % C4) * 4;
                        const int n = nt * BN + cl;
                        if (n >= p.N) continue;
                        int acc4[4] = {0, 0, 0, 0};
                        const int32_t* src = p.ws + (size_t)row_i * p.N + n;
                        const size_t kstride = (size_t)p.M * p.N;
                        if (vec) {
                            int ks = 0;
                            for (; ks + 4 <= p.k_splits; ks += 4) {
                                int4 v[4];
#pragma unroll
                                for (int q = 0; q < 4; ++q) v[q] = __ldcg(reinterpret_cast<const int4*>(src + (ks + q) * kstride));
#pragma unroll
                                for (int q = 0; q < 4; ++q) {
                                    acc4[0] += v[q].x; acc4[1] += v[q].y; acc4[2] += v[q].z; acc4[3] += v[q].w;
                                }
                            }
                            for (; ks < p.k_splits; ++ks) {
                                const int4 v = __ldcg(reinterpret_cast<const int4*>(src + ks * kstride));
                                acc4[0] += v.x; acc4[1] += v.y; acc4[2] += v.z; acc4[3] += v.w;
                            }
                        } else {
                            for (int ks = 0; ks < p.k_splits; ++ks)
#pragma unroll
                                for (int q = 0; q < 4; ++q)
                                    if (n + q < p.N) acc4[q] += __ldcg(src + ks * kstride + q);
                        }
                        const float sa_i = __ldg(p.scale_A + row_i);
                        float* Crow = static_cast<float*>(p.C) + (size_t)row_i * p.N;
                        float o[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            if (n + q < p.N) {
                                const float rs = (EPI == B2_EPI_BIAS_RESIDUAL) ? p.residual[(size_t)row_i * p.N + n + q] : 0.f;
                                o[q] = epilogue<EPI>(acc4[q], sa_i, sB_s[cl + q], EPI != B2_EPI_PLAIN ? bias_s[cl + q] : 0.f, rs);
                            }
                        }
                        if (vec && n + 4 <= p.N) {
                            *reinterpret_cast<float4*>(Crow + n) = make_float4(o[0], o[1], o[2], o[3]);
                        } else {
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                if (n + q < p.N) Crow[n + q] = o[q];
                        }
                    }
                    if (et == 0) *ctr = 0u;  // every k range has arrived: reusable
                }
            }
            named_barrier(2, 128);  // staged columns are free for the next tile
        }
    }

    tc_fence_before();
    __syncthreads();
    // reduce-scatter: no CTA of the cluster exits while a partner may still address its
    // shared memory
    if (p.cluster_k == 2) cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------------ CTA-pair GEMM (cta_group::2)
// For large GEMMs: a cluster of 2 CTAs computes a 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256 split across the pair's TMEM, N = 256). Each CTA loads
// 128 rows of A and 128 of the 256 B rows per stage (32 KB), so an SM moves 2/3 of the
// operand bytes of a 128 x 256 single-CTA tile per MAC, and the ring is 6 stages deep. Both
// CTAs' TMA bytes land on the even CTA's full barrier; the even CTA issues the MMAs and
// commits to both CTAs' barriers; every epilogue warp of the pair releases the even CTA's
// accumulator barrier. No load uses cluster multicast.
constexpr int P2_ROWS = 128;                       // A rows and B rows per CTA per stage
constexpr int P2_STAGE = 2 * P2_ROWS * GM_BK;      // 32 KB
constexpr int P2_STAGES = 5;
constexpr int P2_BN = 256;                         // accumulator columns per CTA
constexpr int P2_OFF_BAR = P2_STAGES * P2_STAGE;
constexpr int P2_NBAR = 2 * P2_STAGES + 5;  // full[S], empty[S], acc_full[2], acc_empty[2], drain
constexpr int P2_OFF_COL = P2_OFF_BAR + P2_NBAR * 8 + 16;
// 8 epilogue warps (2-9): warp w reads TMEM lanes 32 (w % 4) .. +32 (its quadrant), warps 2-5
// columns 0-127 and warps 6-9 columns 128-255 of the accumulator
constexpr int P2_EPI_WARPS = 8;
constexpr int P2_THREADS = (2 + P2_EPI_WARPS) * 32;
// epilogue staging: per epilogue warp one buffer of 32 rows x 32 fp32 (128-byte swizzled)
constexpr int P2_OFF_EPI = (P2_OFF_COL + 2 * P2_BN * 4 + 1023) & ~1023;
constexpr int P2_EPI_BUF = 32 * 32 * 4;
constexpr int P2_SMEM = P2_OFF_EPI + P2_EPI_WARPS * P2_EPI_BUF + 1024;
constexpr uint32_t P2_TMEM_COLS = 2 * P2_BN;

template <int EPI, bool S32>
__global__ void __launch_bounds__(P2_THREADS, 1)
int8_gemm_tc2_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                     const __grid_constant__ CUtensorMap mapC, const GemmParams p, const int c_tma) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + P2_OFF_BAR;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (P2_STAGES + s); };
    auto accf_bar = [&](int a) { return bar0 + 8u * (2 * P2_STAGES + a); };
    auto acce_bar = [&](int a) { return bar0 + 8u * (2 * P2_STAGES + 2 + a); };
    const uint32_t drain_bar = bar0 + 8u * (2 * P2_STAGES + 4);  // the MMA issuer's drain after an abort
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + P2_OFF_BAR + P2_NBAR * 8);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int nk = (p.K + GM_BK - 1) / GM_BK;
    const int m_tiles = (p.M + 2 * P2_ROWS - 1) / (2 * P2_ROWS);
    const int n_tiles = (p.N + P2_BN - 1) / P2_BN;
    const int num_tiles = m_tiles * n_tiles;

    if (threadIdx.x == 0) {
        prefetch_tensormap(&mapA);
        prefetch_tensormap(&mapB);
        for (int s = 0; s < P2_STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(accf_bar(a), 1);
            mbar_init(acce_bar(a), 2 * P2_EPI_WARPS);  // epilogue warps x 2 CTAs
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(const_cast<uint32_t*>(tmem_slot)), P2_TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers are initialised before any remote arrival
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    griddep_wait();
    griddep_launch();

    if (warp == 0) {
        if (lane == 0) {
            const uint64_t pol = policy_evict_last();
            int it = 0;
            for (int t = pair; t < num_tiles && !*abort_flag; t += npairs) {
                int mt, nt;
                tile_coords(t, m_tiles, n_tiles, mt, nt);
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % P2_STAGES;
                    if (it >= P2_STAGES) {
                        if (*abort_flag || !mbar_wait(empty_bar(s), ((it / P2_STAGES) - 1) & 1, p.err)) {
                            *abort_flag = 1;
                            break;
                        }
                    }
                    const uint32_t a_s = sbase + s * P2_STAGE;
                    const uint32_t b_s = a_s + P2_ROWS * GM_BK;
                    if (rank == 0) mbar_arrive_expect_tx(full_bar(s), 2 * P2_STAGE);  // both CTAs' bytes
                    const uint32_t lead_full = mapa_shared(full_bar(s), 0);
                    tma_load_2d_pair(a_s, &mapA, kb * GM_BK, mt * 2 * P2_ROWS + (int)rank * P2_ROWS, lead_full, pol);
                    tma_load_2d_pair(b_s, &mapB, kb * GM_BK, nt * P2_BN + (int)rank * P2_ROWS, lead_full, pol);
                }
            }
            if (rank == 0) {
                // drain: the even CTA's full barriers count both CTAs' bytes, so its last
                // fill of every stage landing covers the pair (the closing cluster barrier
                // keeps the odd CTA resident until then)
                for (int j = max(0, it - P2_STAGES); j < it; ++j)
                    mbar_wait_drain(full_bar(j % P2_STAGES), (j / P2_STAGES) & 1);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_i8(2 * P2_ROWS, P2_BN);
            int it = 0, j = 0;
            for (int t = pair; t < num_tiles && !*abort_flag; t += npairs, ++j) {
                const int a = j & 1, u = j >> 1;
                if (u >= 1 && !mbar_wait(acce_bar(a), (u - 1) & 1, p.err)) { *abort_flag = 1; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem + a * P2_BN;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % P2_STAGES;
                    if (*abort_flag || !mbar_wait(full_bar(s), (it / P2_STAGES) & 1, p.err)) {
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_s = sbase + s * P2_STAGE;
                    const uint64_t da = smem_desc_sw128(a_s);
                    const uint64_t db = smem_desc_sw128(a_s + P2_ROWS * GM_BK);
#pragma unroll
                    for (int k = 0; k < GM_BK / 32; ++k)
                        mma_i8_pair(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
                    mma_commit_pair(mapa_shared(empty_bar(s), 0));
                    mma_commit_pair(mapa_shared(empty_bar(s), 1));
                }
                mma_commit_pair(mapa_shared(accf_bar(a), 0));
                mma_commit_pair(mapa_shared(accf_bar(a), 1));
            }
            if (*abort_flag) {  // drain: every MMA issued has finished before TMEM is freed
                mma_commit_pair(mapa_shared(drain_bar, 0));
                mbar_wait_drain(drain_bar, 0);
            }
        }
        __syncwarp();
    } else {
        constexpr int NE = P2_EPI_WARPS * 32;
        const int quad = warp & 3;
        const int half = (warp - 2) >> 2;  // column half of the accumulator
        const int et = threadIdx.x - 64;
        float* sB_s = reinterpret_cast<float*>(smem + P2_OFF_COL);
        float* bias_s = sB_s + P2_BN;
        const uint32_t lead_acce0 = mapa_shared(acce_bar(0), 0), lead_acce1 = mapa_shared(acce_bar(1), 0);
        unsigned char* buf = smem + P2_OFF_EPI + (warp - 2) * P2_EPI_BUF;
        int j = 0;
        for (int t = pair; t < num_tiles; t += npairs, ++j) {
            const int a = j & 1, u = j >> 1;
            int mt, nt;
            tile_coords(t, m_tiles, n_tiles, mt, nt);
            if constexpr (!S32) {
                for (int c = et; c < P2_BN; c += NE) {
                    const int n = nt * P2_BN + c;
                    sB_s[c] = n < p.N ? __ldg(p.scale_B + n) : 0.f;
                    if (EPI != B2_EPI_PLAIN) bias_s[c] = n < p.N ? __ldg(p.bias + n) : 0.f;
                }
            }
            named_barrier(2, NE);
            const bool ok = !*abort_flag && mbar_wait(accf_bar(a), u & 1, p.err);
            if (!ok) *abort_flag = 1;
            tc_fence_after();
            const int row = mt * 2 * P2_ROWS + (int)rank * P2_ROWS + quad * 32 + lane;
            const bool row_ok = ok && row < p.M;
            const float sa = (!S32 && row_ok) ? __ldg(p.scale_A + row) : 0.f;
            const uint32_t tbase = tmem + a * P2_BN + ((uint32_t)(quad * 32) << 16);
            const int row0 = mt * 2 * P2_ROWS + (int)rank * P2_ROWS + quad * 32;  // this warp's first row
            // 32-column chunks c0 = 8 half .. 8 half + 7 (in 16-column units): the next chunk's
            // TMEM load is in flight while this one is converted and stored
            constexpr int NCH = P2_BN / 32 / 2;  // chunks per warp
            uint32_t r[2][2][16];
            tmem_ld16(tbase + (uint32_t)(half * NCH * 32), r[0][0]);
            tmem_ld16(tbase + (uint32_t)(half * NCH * 32 + 16), r[0][1]);
            tmem_ld_wait();
#pragma unroll
            for (int k = 0; k < NCH; ++k) {
                const int cc = half * NCH + k;  // 32-column chunk index in the tile
                if (k + 1 < NCH) {
                    tmem_ld16(tbase + (uint32_t)((cc + 1) * 32), r[(k + 1) & 1][0]);
                    tmem_ld16(tbase + (uint32_t)((cc + 1) * 32 + 16), r[(k + 1) & 1][1]);
                }
                uint32_t (&rc)[2][16] = r[k & 1];
                const int n = nt * P2_BN + cc * 32;
                float rs[2][16];
#pragma unroll
                for (int i = 0; i < 16; ++i) { rs[0][i] = 0.f; rs[1][i] = 0.f; }
                if constexpr (EPI == B2_EPI_BIAS_RESIDUAL && !S32) {
                    if (row_ok && n < p.N) load_res16(p, row, n, rs[0]);
                    if (row_ok && n + 16 < p.N) load_res16(p, row, n + 16, rs[1]);
                }
                if (c_tma) {
                    // 32 x 32 block of this warp through swizzled shared memory, stored by TMA
                    // (rows >= M and columns >= N are clipped by the tensor map)
                    if (lane == 0) bulk_wait_read<0>();  // the buffer's previous store has read it
                    __syncwarp();
                    uint32_t w[32];
#pragma unroll
                    for (int q = 0; q < 32; ++q) {
                        if constexpr (S32) {
                            w[q] = rc[q >> 4][q & 15];
                        } else {
                            w[q] = __float_as_uint(epilogue<EPI>((int32_t)rc[q >> 4][q & 15], sa, sB_s[cc * 32 + q],
                                                                 EPI != B2_EPI_PLAIN ? bias_s[cc * 32 + q] : 0.f,
                                                                 rs[q >> 4][q & 15]));
                        }
                    }
#pragma unroll
                    for (int ch = 0; ch < 8; ++ch)
                        *reinterpret_cast<uint4*>(buf + lane * 128 + ((ch ^ (lane & 7)) * 16)) =
                            make_uint4(w[4 * ch], w[4 * ch + 1], w[4 * ch + 2], w[4 * ch + 3]);
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0 && ok) {
                        tma_store_2d(&mapC, smem_u32(buf), n, row0);
                        bulk_commit();
                    }
                } else {
                    if (row_ok && n < p.N)
                        store16<EPI, S32>(rc[0], row, n, sa, sB_s + cc * 32, bias_s + cc * 32, rs[0], p);
                    if (row_ok && n + 16 < p.N)
                        store16<EPI, S32>(rc[1], row, n + 16, sa, sB_s + cc * 32 + 16, bias_s + cc * 32 + 16,
                                          rs[1], p);
                }
                tmem_ld_wait();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(a ? lead_acce1 : lead_acce0);
            named_barrier(2, NE);
        }
    }
    if (warp >= 2 && lane == 0) bulk_wait_all();  // epilogue stores complete before exit
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the even CTA's last commits target this CTA's barriers
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, P2_TMEM_COLS);
    }
}

// ------------------------------------------------------------------ SIMT path for K % 16 != 0
// (the tensor-map row stride must be a multiple of 16 bytes). Plain exact int32 dot products.
template <int EPI, bool S32>
__global__ void __launch_bounds__(256)
int8_gemm_simt_kernel(const int32_t* __restrict__ A, const int32_t* __restrict__ BT, const GemmParams p) {
    griddep_wait();
    griddep_launch();
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const int m = blockIdx.y;
    if (n >= p.N) return;
    const int K4 = p.K >> 2;
    const int32_t* a = A + (size_t)m * K4;
    const int32_t* bb = BT + (size_t)n * K4;
    int acc = 0;
    for (int k = 0; k < K4; ++k) acc = __dp4a(a[k], bb[k], acc);
    if constexpr (S32) {
        static_cast<int32_t*>(p.C)[(size_t)m * p.N + n] = acc;
    } else {
        const float bi = (EPI != B2_EPI_PLAIN) ? p.bias[n] : 0.f;
        const float rs = (EPI == B2_EPI_BIAS_RESIDUAL) ? p.residual[(size_t)m * p.N + n] : 0.f;
        static_cast<float*>(p.C)[(size_t)m * p.N + n] = epilogue<EPI>(acc, p.scale_A[m], p.scale_B[n], bi, rs);
    }
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

// int8 row-major [rows, K] operand, box = box_rows x 128 bytes, 128-byte swizzle.
static bool encode_map(CUtensorMap* map, const void* base, int rows, int K, int box_rows) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)K};
    cuuint32_t box[2] = {(cuuint32_t)GM_BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Small cache of encoded tensor maps (decode loops call the same weights every step).
static bool make_map(CUtensorMap* map, const void* base, int rows, int K, int box_rows) {
    struct Entry { int dev; const void* base; int rows, K, box; CUtensorMap map; };
    constexpr int kEntries = 64;
    static Entry cache[kEntries];
    static int fill = 0, next = 0;
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    for (int i = 0; i < fill; ++i) {
        const Entry& e = cache[i];
        if (e.dev == dev && e.base == base && e.rows == rows && e.K == K && e.box == box_rows) {
            *map = e.map;
            return true;
        }
    }
    if (!encode_map(map, base, rows, K, box_rows)) return false;
    Entry& e = cache[next];
    e = Entry{dev, base, rows, K, box_rows, *map};
    next = (next + 1) % kEntries;
    if (fill < kEntries) ++fill;
    return true;
}

int num_sms_current_device();
bool set_smem_attr_once(const void* func, int bytes, int slot);

template <int BN, int EPI, bool S32>
static int launch_tc(const GemmParams& p, const int32_t* A, const int32_t* BT, cudaStream_t st, int slot) {
    using C = GemmCfg<BN>;
    CUtensorMap ma, mb;
    if (!make_map(&ma, A, p.M, p.K, p.a_rows) || !make_map(&mb, BT, p.N, p.K, BN)) return B2_ERR_CUDA;
    auto kfn = int8_gemm_tc_kernel<BN, EPI, S32>;
    if (!set_smem_attr_once((const void*)kfn, C::SMEM, slot)) return B2_ERR_CUDA;
    const int tiles = ((p.N + BN - 1) / BN) * ((p.M + GM_BM - 1) / GM_BM);
    const int grid = std::min(tiles * p.k_splits, num_sms_current_device());
    if (p.cluster_k) {  // one CTA per (tile, k range); a tile's k ranges form a cluster
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(tiles * p.k_splits);
        cfg.blockDim = dim3(GM_THREADS);
        cfg.dynamicSmemBytes = C::SMEM;
        cfg.stream = st;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = p.k_splits;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl_enabled() ? 2 : 1;
        return cudaLaunchKernelEx(&cfg, kfn, ma, mb, p) == cudaSuccess ? B2_OK : B2_ERR_CUDA;
    }
    return launch_kernel(kfn, dim3(grid), dim3(GM_THREADS), (size_t)C::SMEM, st, ma, mb, p) == cudaSuccess
               ? B2_OK
               : B2_ERR_CUDA;
}

// CTA-pair path switch (a test hook compares it with the single-CTA path).
bool g_gemm_pairs = true;

// Split-K plan for GEMMs whose tiles cannot fill the GPU (decode: M = batch <= 128): the
// workspace holds [tiles] u32 tickets (zero at rest), then [k_splits][M][N] int32 partials.
static void plan_split(GemmParams& p, int tiles, void* ws, size_t ws_bytes, int sms) {
    p.cluster_k = 0;
    p.k_splits = 1;
    p.kb_per_split = (p.K + GM_BK - 1) / GM_BK;
    p.ws = nullptr;
    p.counters = nullptr;
    const int nk = p.kb_per_split;
    if (!ws || tiles >= sms || nk < 2) return;
    int ks = std::min(std::min(nk, sms / std::max(1, tiles)), 32);
    if (ks < 2) return;
    const int kbps = (nk + ks - 1) / ks;
    ks = (nk + kbps - 1) / kbps;
    const size_t ctr_bytes = (((size_t)tiles * sizeof(unsigned int)) + 255) & ~(size_t)255;
    const size_t need = ctr_bytes + (size_t)ks * p.M * p.N * sizeof(int32_t);
    if (ks < 2 || need > ws_bytes) return;
    p.k_splits = ks;
    p.kb_per_split = kbps;
    p.counters = static_cast<unsigned int*>(ws);
    p.ws = reinterpret_cast<int32_t*>(static_cast<char*>(ws) + ctr_bytes);
}

template <int EPI, bool S32>
static int launch_tc2(const GemmParams& p, const int32_t* A, const int32_t* BT, cudaStream_t st, int slot) {
    CUtensorMap ma, mb, mc;
    if (!make_map(&ma, A, p.M, p.K, P2_ROWS) || !make_map(&mb, BT, p.N, p.K, P2_ROWS)) return B2_ERR_CUDA;
    // fp32 / int32 output map with 32 x 32 boxes in the 128-byte swizzle, when the row pitch
    // and base allow TMA (else the kernel stores directly)
    int c_tma = ((p.N & 3) == 0 && ((uintptr_t)p.C & 15) == 0) ? 1 : 0;
    if (c_tma) {
        EncodeTiledFn enc = get_encode_fn();
        cuuint64_t dims[2] = {(cuuint64_t)p.N, (cuuint64_t)p.M};
        cuuint64_t strides[1] = {(cuuint64_t)p.N * 4};
        cuuint32_t box[2] = {32, 32};
        cuuint32_t estr[2] = {1, 1};
        c_tma = enc && enc(&mc, S32 ? CU_TENSOR_MAP_DATA_TYPE_INT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, p.C, dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    if (!c_tma) memset(&mc, 0, sizeof(mc));
    auto kfn = int8_gemm_tc2_kernel<EPI, S32>;
    if (!set_smem_attr_once((const void*)kfn, P2_SMEM, slot)) return B2_ERR_CUDA;
    const int tiles = ((p.N + P2_BN - 1) / P2_BN) * ((p.M + 2 * P2_ROWS - 1) / (2 * P2_ROWS));
    const int pairs = std::min(tiles, num_sms_current_device() / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(P2_THREADS);
    cfg.dynamicSmemBytes = P2_SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kfn, ma, mb, mc, p, c_tma) == cudaSuccess ? B2_OK : B2_ERR_CUDA;
}

constexpr int kMaxGemmDevices = 64;

// Clusters of c CTAs of the 128-column kernel that the device holds at once (cached).
template <int EPI, bool S32>
static int rs_resident_clusters(int c) {
    static int cached[4][kMaxGemmDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxGemmDevices) return 0;
    const int ci = c == 2 ? 0 : c == 4 ? 1 : 2;
    if (cached[ci][dev]) return cached[ci][dev] - 1;
    auto kfn = int8_gemm_tc_kernel<128, EPI, S32>;
    int n = 0;
    if (set_smem_attr_once((const void*)kfn, GemmCfg<128>::SMEM, 0)) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(c);
        cfg.blockDim = dim3(GM_THREADS);
        cfg.dynamicSmemBytes = GemmCfg<128>::SMEM;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = c;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
    }
    cached[ci][dev] = n + 1;
    return n;
}

// Cluster size of the reduce-scatter split (GemmParams::cluster_k == 2) for a decode
// contraction, or 1. With one 128-row tile, the 32-column path streams the whole activation
// through every one of its CTAs (config-5 shard 128 x 4096 x 4096: 128 CTAs x 512 KB of A
// for 16 MB of weights, ~10 us of TMA per CTA); 128-column tiles whose K range is split over
// a cluster of c CTAs stream A[:, k range] once per (tile, k range) instead, 4x less at the
// same CTA count, and exchange (c - 1) / c of a 128 x 128 int32 partial through L2.
// Used once the activation holds >= 256 KB (B2_GEMM_RS_MIN_KB sets the bound in KB,
// B2_GEMM_RS=0 turns it off), with every cluster resident at once (a second wave of
// clusters doubles the time), >= 4 k-blocks per CTA and no empty k range.
template <int EPI, bool S32>
static int rs_cluster_size(const GemmParams& p, int sms) {
    static const bool off = getenv("B2_GEMM_RS") && strcmp(getenv("B2_GEMM_RS"), "0") == 0;
    static const long long min_a = (getenv("B2_GEMM_RS_MIN_KB") ? atoll(getenv("B2_GEMM_RS_MIN_KB")) : 256) * 1024;
    if (off || p.M > GM_BM || (long long)p.a_rows * p.K < min_a) return 1;
    const int t128 = (p.N + 127) / 128;
    const int nk = (p.K + GM_BK - 1) / GM_BK;
    for (int c = 8; c >= 2; c /= 2) {
        const int kbps = (nk + c - 1) / c;
        if (t128 * c > sms || kbps < 4 || (c - 1) * kbps >= nk) continue;
        if (t128 > rs_resident_clusters<EPI, S32>(c)) continue;
        return c;
    }
    return 1;
}

// Exchange bytes of the reduce-scatter split: (c - 1) 128 x (128 / c) int32 slices per
// (tile, owner).
static size_t rs_ws_bytes(int N, int c) {
    return (size_t)((N + 127) / 128) * (c - 1) * GM_BM * 128 * sizeof(int32_t);
}

static void set_rs_split(GemmParams& p, int c, void* ws) {
    const int nk = (p.K + GM_BK - 1) / GM_BK;
    p.k_splits = c;
    p.kb_per_split = (nk + c - 1) / c;
    p.cluster_k = 2;
    p.ws = static_cast<int32_t*>(ws);
    p.counters = nullptr;
}

template <int EPI, bool S32>
static int gemm_dispatch(GemmParams& p, const int32_t* A, const int32_t* BT, void* ws, size_t ws_bytes,
                         cudaStream_t st) {
    // K == 0 (empty contraction, acc = 0) and K % 16 != 0 take the SIMT kernel
    if (p.K == 0 || (p.K & 15) != 0 || ((uintptr_t)A & 15) || ((uintptr_t)BT & 15)) {
        dim3 grid((p.N + 255) / 256, p.M);
        return launch_kernel(int8_gemm_simt_kernel<EPI, S32>, grid, dim3(256), 0, st, A, BT, p) == cudaSuccess
                   ? B2_OK
                   : B2_ERR_CUDA;
    }
    const int sms = num_sms_current_device();
    const int mt = (p.M + GM_BM - 1) / GM_BM;
    // widest tile that still gives every SM a tile; otherwise the narrowest, split along K
    const int slot_base = (EPI + (S32 ? 4 : 0)) * 3;
    const int t256 = mt * ((p.N + 255) / 256), t128 = mt * ((p.N + 127) / 128), t64 = mt * ((p.N + 63) / 64);
    // CTA pairs with 256 x 256 tiles once there are enough of them to occupy most SM pairs
    const int pair_tiles = ((p.M + 255) / 256) * ((p.N + 255) / 256);
    if (g_gemm_pairs && pair_tiles * 2 >= (sms * 3) / 4) {
        plan_split(p, pair_tiles, nullptr, 0, sms);
        return launch_tc2<EPI, S32>(p, A, BT, st, 40 + EPI + (S32 ? 4 : 0));
    }
    if (t256 >= sms) {
        plan_split(p, t256, nullptr, 0, sms);
        return launch_tc<256, EPI, S32>(p, A, BT, st, slot_base + 0);
    }
    if (t128 >= sms) {
        plan_split(p, t128, nullptr, 0, sms);
        return launch_tc<128, EPI, S32>(p, A, BT, st, slot_base + 1);
    }
    if (const int rc = rs_cluster_size<EPI, S32>(p, sms); rc > 1 && ws && ws_bytes >= rs_ws_bytes(p.N, rc)) {
        set_rs_split(p, rc, ws);
        return launch_tc<128, EPI, S32>(p, A, BT, st, slot_base + 1);
    }
    // skinny outputs (decode: M = batch): 32-column tiles double the CTAs streaming the weights
    const int t32 = mt * ((p.N + 31) / 32);
    if (!ws && t64 * 2 <= sms && t32 <= sms) {
        plan_split(p, t32, nullptr, 0, sms);
        // Long contractions (decode FC2: K = 3072) split K over a cluster of 2 or 4 CTAs per
        // tile, each keeping >= 6 k-blocks, whose int32 partials meet in rank 0's shared
        // memory: the chain of MMA issues per CTA shrinks with the split (FC2 64x768x3072:
        // 9.7 -> 6.8 us; 8 CTAs no faster; splitting K = 768 into 2 or 4 measured slower,
        // 4.4 -> 5.1 us, the partial exchange then outweighing 3 k-blocks of MMAs).
        static const bool cluster_off = getenv("B2_GEMM_CLUSTER") && strcmp(getenv("B2_GEMM_CLUSTER"), "0") == 0;
        const int nk = (p.K + GM_BK - 1) / GM_BK;
        int ks = 1;
        for (int c = GemmCfg<32>::RED_MAX + 1; c >= 2; c /= 2)
            if (nk >= 6 * c && t32 * c <= sms) { ks = c; break; }
        if (!cluster_off && ks > 1 && !p.sc.q && p.k_splits == 1) {
            p.k_splits = ks;
            p.kb_per_split = (nk + ks - 1) / ks;
            p.cluster_k = 1;
        }
        return launch_tc<32, EPI, S32>(p, A, BT, st, 48 + EPI + (S32 ? 4 : 0));
    }
    plan_split(p, t64, S32 ? nullptr : ws, ws_bytes, sms);  // the raw-int32 view is never split
    return launch_tc<64, EPI, S32>(p, A, BT, st, slot_base + 2);
}

// Exchange bytes the reduce-scatter split needs for this shape (0 when gemm_launch would take
// another path: CTA pairs, a tile per SM, or a small activation).
size_t gemm_rs_workspace_size(int M, int N, int K) {
    if (M <= 0 || N <= 0 || K <= 0 || (K & 15)) return 0;
    const int sms = num_sms_current_device();
    const int mt = (M + GM_BM - 1) / GM_BM;
    const int pair_tiles = ((M + 255) / 256) * ((N + 255) / 256);
    if ((g_gemm_pairs && pair_tiles * 2 >= (sms * 3) / 4) || mt * ((N + 255) / 256) >= sms ||
        mt * ((N + 127) / 128) >= sms)
        return 0;
    GemmParams p{};
    p.M = M;
    p.N = N;
    p.K = K;
    p.a_rows = M <= GM_BM ? ((M + 7) & ~7) : GM_BM;
    const int rc = rs_cluster_size<B2_EPI_PLAIN, false>(p, sms);
    return rc > 1 ? rs_ws_bytes(N, rc) : 0;
}

// Workspace bytes that let gemm_launch split K for these shapes (0 when it would not split).
size_t gemm_workspace_size(int M, int N, int K) {
    const int sms = num_sms_current_device();
    const int mt = (M + GM_BM - 1) / GM_BM;
    const int tiles = mt * ((N + 63) / 64);
    const int nk = (K + GM_BK - 1) / GM_BK;
    if (mt * ((N + 127) / 128) >= sms || nk < 2) return 0;
    size_t need = 0;
    if (tiles < sms) {
        const size_t ctr_bytes = (((size_t)tiles * sizeof(unsigned int)) + 255) & ~(size_t)255;
        need = ctr_bytes + (size_t)std::min(std::min(nk, sms / std::max(1, tiles)), 32) * M * N * sizeof(int32_t);
    }
    return std::max(need, gemm_rs_workspace_size(M, N, K));
}

int gemm_launch(int M, int N, int K, const int32_t* A, const int32_t* BT, const float* sA, const float* sB,
                const float* bias, const float* residual, void* C, int epi, bool s32, cudaStream_t st,
                void* ws, size_t ws_bytes) {
    if (M < 0 || N < 0 || K < 0 || (K & 3)) return B2_ERR_INVALID;
    if (M == 0 || N == 0) return B2_OK;
    if (!A || !BT || !C) return B2_ERR_INVALID;
    if (!s32) {
        if (!sA || !sB) return B2_ERR_INVALID;
        if (epi < B2_EPI_PLAIN || epi > B2_EPI_BIAS_RESIDUAL) return B2_ERR_INVALID;
        if (epi != B2_EPI_PLAIN && !bias) return B2_ERR_INVALID;
        if (epi == B2_EPI_BIAS_RESIDUAL && !residual) return B2_ERR_INVALID;
    }
    GemmParams p{M, N, K, sA, sB, bias, residual, C, device_error_ptr(), 1, 0, nullptr, nullptr,
                 M <= GM_BM ? ((M + 7) & ~7) : GM_BM};
    p.b_early = weights_constant() ? 1 : 0;
    if (s32) return gemm_dispatch<B2_EPI_PLAIN, true>(p, A, BT, ws, ws_bytes, st);
    switch (epi) {
        case B2_EPI_PLAIN: return gemm_dispatch<B2_EPI_PLAIN, false>(p, A, BT, ws, ws_bytes, st);
        case B2_EPI_BIAS: return gemm_dispatch<B2_EPI_BIAS, false>(p, A, BT, ws, ws_bytes, st);
        case B2_EPI_BIAS_GELU: return gemm_dispatch<B2_EPI_BIAS_GELU, false>(p, A, BT, ws, ws_bytes, st);
        default: return gemm_dispatch<B2_EPI_BIAS_RESIDUAL, false>(p, A, BT, ws, ws_bytes, st);
    }
}

// The engine's QKV linear with the split into q and the paged K/V write fused into the
// epilogue (bias epilogue, then the 16-column stores go to q or the cache row of pos[b]).
// Only the one-CTA tcgen05 kernel implements it; shapes that would take another kernel (or
// N != 3 d, d % 16 != 0) return B2_ERR_UNSUPPORTED and the caller runs the two steps apart.
int gemm_launch_qkv(int M, int N, int K, const int32_t* A, const int32_t* BT, const float* sA, const float* sB,
                    const float* bias, const QkvScatterArgs& sc, cudaStream_t st, void* ws, size_t ws_bytes) {
    if (M <= 0 || N <= 0 || (K & 15) || K == 0 || ((uintptr_t)A & 15) || ((uintptr_t)BT & 15)) return B2_ERR_UNSUPPORTED;
    if (!A || !BT || !sA || !sB || !bias || !sc.q || !sc.k || !sc.v || !sc.pos || !sc.block_table)
        return B2_ERR_INVALID;
    if (sc.d <= 0 || sc.d % 16 || N != 3 * sc.d || M > GM_BM) return B2_ERR_UNSUPPORTED;
    GemmParams p{M, N, K, sA, sB, bias, nullptr, sc.q, device_error_ptr(), 1, 0, nullptr, nullptr, (M + 7) & ~7};
    p.b_early = weights_constant() ? 1 : 0;
    p.sc.q = sc.q;
    p.sc.k = sc.k;
    p.sc.v = sc.v;
    p.sc.pos = sc.pos;
    p.sc.block_table = sc.block_table;
    p.sc.d = sc.d;
    p.sc.bs = sc.block_size;
    p.sc.nbps = sc.nbps;
    p.sc.bf16 = sc.bf16;
    // the tile choice of gemm_dispatch for M <= 128 outside the CTA-pair range
    const int sms = num_sms_current_device();
    const int pair_tiles = (N + 255) / 256;
    if (g_gemm_pairs && pair_tiles * 2 >= (sms * 3) / 4) return B2_ERR_UNSUPPORTED;
    const int t256 = (N + 255) / 256, t128 = (N + 127) / 128, t64 = (N + 63) / 64, t32 = (N + 31) / 32;
    plan_split(p, 1, nullptr, 0, sms);  // one k range per tile (sets kb_per_split)
    if (t256 >= sms) return launch_tc<256, B2_EPI_BIAS, false>(p, A, BT, st, 0);
    if (t128 >= sms) return launch_tc<128, B2_EPI_BIAS, false>(p, A, BT, st, 0);
    if (const int rc = rs_cluster_size<B2_EPI_BIAS, false>(p, sms); rc > 1 && ws && ws_bytes >= rs_ws_bytes(N, rc)) {
        set_rs_split(p, rc, ws);
        return launch_tc<128, B2_EPI_BIAS, false>(p, A, BT, st, 0);
    }
    if (t64 * 2 <= sms && t32 <= sms) return launch_tc<32, B2_EPI_BIAS, false>(p, A, BT, st, 0);
    return launch_tc<64, B2_EPI_BIAS, false>(p, A, BT, st, 0);
}

}  // namespace b2
