// Tied vocab projection + greedy argmax on tcgen05, for the batched decode step.
//
// The reference computes logits[v] = sum_k h[k] wte[v,k] in fp32 on CUDA cores, one thread per
// vocab row (src/gpt2_engine.cu:391-403), then copies all logits to the host for argmax
// (src/sampler.cu:10-14). At batch 64-128 that is 5-53 GFLOP per step, which CUDA cores need
// 70-730 us for. Here both operands are split into bf16 pairs, x = hi + lo with
// hi = bf16(x), lo = bf16(x - hi) (16 significant bits), and three tensor-core products
// hi.hi + hi.lo + lo.hi accumulate in fp32 TMEM: each term carries a relative error of about
// 2^-16, far below the spacing of distinct logits, at tensor-core speed; the step stays
// HBM-bound on the 2 x V x d bf16 embedding halves.
//
// Kernel (persistent, 192 threads, one CTA per SM): warp 0 TMA-loads 128 x 64 bf16 tiles of
// h_hi/h_lo and BN x 64 tiles of wte_hi/wte_lo (128-byte swizzle) into a 3-stage ring; warp 1
// issues tcgen05.mma.kind::f16 (bf16 x bf16 -> fp32, M=128, N=BN, K=16) three times per
// 16-wide K step; warps 2-5 read the accumulator (thread = batch row), optionally store the
// logits, and fold the tile's maximum into a per-row 64-bit atomicMax key ordered by value
// then lowest index (the reference's std::max_element tie rule).
#include "common.cuh"
#include <cuda_bf16.h>
#include <algorithm>
#include <mutex>

namespace b2 {

int num_sms_current_device();
bool set_smem_attr_once(const void* func, int bytes, int slot);

constexpr int VT_BM = 128, VT_BN = 128, VT_BKB = 128;  // BK in bytes = 64 bf16
constexpr int VT_THREADS = 192;
constexpr int VT_A = VT_BM * VT_BKB, VT_B = VT_BN * VT_BKB;
constexpr int VT_STAGE = 2 * VT_A + 2 * VT_B;  // A_hi, A_lo, W_hi, W_lo
constexpr int VT_STAGES = 3;
constexpr int VT_OFF_BAR = VT_STAGES * VT_STAGE;
constexpr int VT_NBAR = 2 * VT_STAGES + 5;  // full[S], empty[S], acc_full[2], acc_empty[2], drain
constexpr int VT_OFF_XP = VT_OFF_BAR + 256;          // epilogue transpose blocks, one per epilogue warp
constexpr int VT_XP_LD = 33;                          // padded row of a 32 x 32 fp32 block
constexpr int VT_SMEM = VT_OFF_XP + 4 * 32 * VT_XP_LD * 4 + 1024;
constexpr uint32_t VT_ACC_COLS = VT_BN, VT_TMEM_COLS = 2 * VT_BN;

__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4)                       // D format: f32
         | (1u << 7)                       // A format: bf16
         | (1u << 10)                      // B format: bf16
         | ((uint32_t)(N >> 3) << 17)
         | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}

__device__ __forceinline__ unsigned long long vt_key(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}

struct VocabParams {
    int M, N, K;               // batch, vocab rows held here, d_model
    int n_offset;              // global index of this shard's first vocab row (tensor parallel)
    int a_rows;                // rows of the activation tiles each stage loads (M rounded to 8, <= 128)
    float* logits;             // [M, N] or null
    unsigned long long* keys;  // [M] argmax keys (reset by the caller before the step)
    unsigned int* err;
    // argmax candidates for the exact rescoring (null: none recorded): every logit within
    // delta of its row's running maximum, as (value bits, local vocab index) pairs
    float delta;
    int* cand_cnt;             // [M] (reset by the caller before the step)
    int2* cand;                // [M, cand_cap]
    int cand_cap;
};

__global__ void __launch_bounds__(VT_THREADS, 1)
vocab_bf16x3_kernel(const __grid_constant__ CUtensorMap mAh, const __grid_constant__ CUtensorMap mAl,
                    const __grid_constant__ CUtensorMap mWh, const __grid_constant__ CUtensorMap mWl,
                    const VocabParams p) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + VT_OFF_BAR;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (VT_STAGES + s); };
    auto accf_bar = [&](int a) { return bar0 + 8u * (2 * VT_STAGES + a); };
    auto acce_bar = [&](int a) { return bar0 + 8u * (2 * VT_STAGES + 2 + a); };
    const uint32_t drain_bar = bar0 + 8u * (2 * VT_STAGES + 4);  // the MMA issuer's drain after an abort
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + VT_OFF_BAR + VT_NBAR * 8);
    volatile uint32_t* abort_flag = tmem_slot + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = (p.K * 2 + VT_BKB - 1) / VT_BKB;  // 64-element K blocks
    const int m_tiles = (p.M + VT_BM - 1) / VT_BM;
    const int n_tiles = (p.N + VT_BN - 1) / VT_BN;
    const int num_tiles = m_tiles * n_tiles;

    if (threadIdx.x == 0) {
        prefetch_tensormap(&mAh); prefetch_tensormap(&mAl);
        prefetch_tensormap(&mWh); prefetch_tensormap(&mWl);
        for (int s = 0; s < VT_STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(accf_bar(a), 1);
            mbar_init(acce_bar(a), 4);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(const_cast<uint32_t*>(tmem_slot)), VT_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // the embedding halves are constant: the first stages' W tiles are requested
            // before waiting on the previous kernel, the activation tiles after
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_a = policy_evict_last();
            int npre = 0;
            if ((int)blockIdx.x < num_tiles) {
                const int nt = blockIdx.x / m_tiles;
                npre = min(VT_STAGES, nk);
                for (int i = 0; i < npre; ++i) {
                    const uint32_t w_s = sbase + i * VT_STAGE + 2 * VT_A;
                    mbar_arrive_expect_tx(full_bar(i), 2 * p.a_rows * VT_BKB + 2 * VT_B);
                    tma_load_2d(w_s, &mWh, i * 64, nt * VT_BN, full_bar(i), pol_w);
                    tma_load_2d(w_s + VT_B, &mWl, i * 64, nt * VT_BN, full_bar(i), pol_w);
                }
            }
            griddep_wait();
            griddep_launch();
            int it = 0;
            for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
                const int mt = t % m_tiles, nt = t / m_tiles;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % VT_STAGES;
                    const uint32_t a_s = sbase + s * VT_STAGE;
                    const uint32_t w_s = a_s + 2 * VT_A;
                    if (it >= npre) {
                        if (it >= VT_STAGES &&
                            (*abort_flag || !mbar_wait(empty_bar(s), ((it / VT_STAGES) - 1) & 1, p.err))) {
                            *abort_flag = 1;
                            break;
                        }
                        mbar_arrive_expect_tx(full_bar(s), 2 * p.a_rows * VT_BKB + 2 * VT_B);
                        tma_load_2d(w_s, &mWh, kb * 64, nt * VT_BN, full_bar(s), pol_w);
                        tma_load_2d(w_s + VT_B, &mWl, kb * 64, nt * VT_BN, full_bar(s), pol_w);
                    }
                    tma_load_2d(a_s, &mAh, kb * 64, mt * VT_BM, full_bar(s), pol_a);
                    tma_load_2d(a_s + VT_A, &mAl, kb * 64, mt * VT_BM, full_bar(s), pol_a);
                }
            }
            // drain: the last fill of every stage this thread requested has landed before the
            // CTA can exit, also when a consumer gave up waiting (a prefetched fill whose
            // activation tiles were never requested cannot complete; its bounded wait covers
            // the embedding tiles in flight)
            for (int j = max(0, it - VT_STAGES); j < max(it, npre); ++j)
                mbar_wait_drain(full_bar(j % VT_STAGES), (j / VT_STAGES) & 1);
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(VT_BM, VT_BN);
            int it = 0, j = 0;
            for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x, ++j) {
                const int a = j & 1, u = j >> 1;
                if (u >= 1 && !mbar_wait(acce_bar(a), (u - 1) & 1, p.err)) { *abort_flag = 1; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem + a * VT_ACC_COLS;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % VT_STAGES;
                    if (*abort_flag || !mbar_wait(full_bar(s), (it / VT_STAGES) & 1, p.err)) {
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_s = sbase + s * VT_STAGE;
                    const uint64_t dah = smem_desc_sw128(a_s), dal = smem_desc_sw128(a_s + VT_A);
                    const uint64_t dwh = smem_desc_sw128(a_s + 2 * VT_A), dwl = smem_desc_sw128(a_s + 2 * VT_A + VT_B);
#pragma unroll
                    for (int k = 0; k < VT_BKB / 32; ++k) {  // 16 bf16 = 32 bytes per MMA
                        const uint32_t first = (kb | k) != 0 ? 1u : 0u;
                        mma_bf16(d_tmem, dah + 2 * k, dwh + 2 * k, idesc, first);
                        mma_bf16(d_tmem, dah + 2 * k, dwl + 2 * k, idesc, 1u);
                        mma_bf16(d_tmem, dal + 2 * k, dwh + 2 * k, idesc, 1u);
                    }
                    mma_commit(empty_bar(s));
                }
                mma_commit(accf_bar(a));
            }
            if (*abort_flag) {  // drain: every MMA issued has finished before TMEM is freed
                mma_commit(drain_bar);
                mbar_wait_drain(drain_bar, 0);
            }
        }
        __syncwarp();
    } else {
        const int quad = warp & 3;
        griddep_wait();
        int j = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++j) {
            const int a = j & 1, u = j >> 1;
            const int mt = t % m_tiles, nt = t / m_tiles;
            const bool ok = !*abort_flag && mbar_wait(accf_bar(a), u & 1, p.err);
            if (!ok) *abort_flag = 1;
            tc_fence_after();
            const int row = mt * VT_BM + quad * 32 + lane;
            const bool row_ok = ok && row < p.M;
            const uint32_t tbase = tmem + a * VT_ACC_COLS + ((uint32_t)(quad * 32) << 16);
            unsigned long long best = 0ull;
            float* xp = reinterpret_cast<float*>(smem + VT_OFF_XP) + quad * 32 * VT_XP_LD;
            const int row0 = mt * VT_BM + quad * 32;
#pragma unroll 1
            for (int c = 0; c < VT_BN / 16; c += 2) {
                uint32_t r0[16], r1[16];
                tmem_ld16(tbase + (uint32_t)(c * 16), r0);
                tmem_ld16(tbase + (uint32_t)(c * 16 + 16), r1);
                tmem_ld_wait();
                const int n0 = nt * VT_BN + c * 16;
                if (!ok) continue;
#pragma unroll
                for (int q = 0; q < 32; ++q) {
                    const int n = n0 + q;
                    const float v = __uint_as_float(q < 16 ? r0[q] : r1[q - 16]);
                    if (row_ok && n < p.N) {
                        const unsigned long long key = vt_key(v, p.n_offset + n);
                        best = key > best ? key : best;
                    }
                    xp[lane * VT_XP_LD + q] = v;
                }
                if (p.logits) {
                    // transposed through shared memory so that each store writes 32 consecutive
                    // logits of one row (128 bytes) instead of one logit of 32 rows
                    __syncwarp();
                    const int n = n0 + lane;
#pragma unroll 4
                    for (int r = 0; r < 32; ++r)
                        if (row0 + r < p.M && n < p.N) p.logits[(size_t)(row0 + r) * p.N + n] = xp[r * VT_XP_LD + lane];
                }
                __syncwarp();
            }
            // the row's running maximum including this tile, then a second pass over the
            // accumulator records every value within delta of it. The running maximum only
            // grows, so whatever ends within delta of the row's final maximum is recorded.
            // (tcgen05.ld is warp-wide: every lane of the warp runs the second pass' loads.)
            float thr = INFINITY;
            if (row_ok && best) {
                const unsigned long long old = atomicMax(p.keys + row, best);
                const unsigned long long m = old > best ? old : best;
                uint32_t mu = (uint32_t)(m >> 32);
                mu = (mu & 0x80000000u) ? (mu & 0x7fffffffu) : ~mu;
                thr = __uint_as_float(mu) - p.delta;
            }
            if (p.cand && __any_sync(0xffffffffu, thr < INFINITY)) {
#pragma unroll 1
                for (int c = 0; c < VT_BN / 16; c += 2) {
                    uint32_t r0[16], r1[16];
                    tmem_ld16(tbase + (uint32_t)(c * 16), r0);
                    tmem_ld16(tbase + (uint32_t)(c * 16 + 16), r1);
                    tmem_ld_wait();
                    const int n0 = nt * VT_BN + c * 16;
#pragma unroll
                    for (int q = 0; q < 32; ++q) {
                        const float v = __uint_as_float(q < 16 ? r0[q] : r1[q - 16]);
                        if (row_ok && n0 + q < p.N && v >= thr) {  // rows past M hold stale products
                            const int i = atomicAdd(p.cand_cnt + row, 1);
                            if (i < p.cand_cap)
                                p.cand[(size_t)row * p.cand_cap + i] = make_int2(__float_as_int(v), n0 + q);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acce_bar(a));
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, VT_TMEM_COLS);
    }
}

// hi = bf16(x), lo = bf16(x - hi) for n values
__global__ void split_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ hi,
                                  __nv_bfloat16* __restrict__ lo, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const __nv_bfloat16 h = __float2bfloat16_rn(x[i]);
        hi[i] = h;
        lo[i] = __float2bfloat16_rn(x[i] - __bfloat162float(h));
    }
}

// ------------------------------------------------------------------ host
typedef CUresult (*EncodeTiledFnV)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static bool encode_bf16(CUtensorMap* map, const void* base, int rows, int K, int box_rows) {
    static EncodeTiledFnV fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return false;
        fn = reinterpret_cast<EncodeTiledFnV>(ptr);
    }
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_split_bf16(const float* x, void* hi, void* lo, size_t n, cudaStream_t st) {
    return launch_kernel(split_bf16_kernel, dim3(592), dim3(256), 0, st, x, static_cast<__nv_bfloat16*>(hi),
                         static_cast<__nv_bfloat16*>(lo), n) == cudaSuccess
               ? B2_OK
               : B2_ERR_CUDA;
}

// logits/argmax of h [M, K] (as bf16 hi/lo) against W [N, K] (bf16 hi/lo). K % 8 == 0.
int launch_vocab_bf16x3(int M, int N, int K, const void* h_hi, const void* h_lo, const void* w_hi, const void* w_lo,
                        float* logits, unsigned long long* keys, cudaStream_t st, int n_offset, float cand_delta,
                        int* cand_cnt, void* cand, int cand_cap) {
    if ((K & 7) || M <= 0 || N <= 0) return B2_ERR_UNSUPPORTED;
    CUtensorMap ah, al, wh, wl;
    // a decode batch loads only its own rows of the activation tiles (the MMA rows past them
    // read stale shared memory and are never stored): half the activation bytes at M = 64
    const int a_rows = M < VT_BM ? ((M + 7) & ~7) : VT_BM;
    if (!encode_bf16(&ah, h_hi, M, K, a_rows) || !encode_bf16(&al, h_lo, M, K, a_rows) ||
        !encode_bf16(&wh, w_hi, N, K, VT_BN) || !encode_bf16(&wl, w_lo, N, K, VT_BN))
        return B2_ERR_CUDA;
    if (!set_smem_attr_once((const void*)vocab_bf16x3_kernel, VT_SMEM, 60)) return B2_ERR_CUDA;
    const int tiles = ((M + VT_BM - 1) / VT_BM) * ((N + VT_BN - 1) / VT_BN);
    VocabParams p{M, N, K, n_offset, a_rows, logits, keys, device_error_ptr(), cand_delta, cand_cnt,
                  static_cast<int2*>(cand), cand_cap};
    const int grid = std::min(tiles, num_sms_current_device());
    return launch_kernel(vocab_bf16x3_kernel, dim3(grid), dim3(VT_THREADS), (size_t)VT_SMEM, st, ah, al, wh, wl, p) ==
                   cudaSuccess
               ? B2_OK
               : B2_ERR_CUDA;
}

}  // namespace b2
