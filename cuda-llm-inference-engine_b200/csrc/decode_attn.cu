// K13 on sm_100a: split-K paged decode attention, one query token per sequence.
//
// Semantics follow the reference's decode_attn_partial_kernel + decode_attn_reduce_kernel
// (kernels/decode/13_decode_attn.cuh:30-189, kernels/decode/13_decode_attn.cu:10-53):
//   O[b,h,:] = softmax(q[b,h] . K[b, 0..ctx_b)^T * scale) . V[b, 0..ctx_b)
// with K/V rows found through the block table, kv_head = h / (H_q / H_kv), and the KV
// sequence split into ranges of whole blocks whose partial (o, m, l) are merged by
// log-sum-exp. It implements the intended math where the reference does not: empty
// splits contribute nothing (the reference leaves their workspace rows unwritten and then
// reads them, 13_decode_attn.cuh:56), a zero-length context yields O = 0, head_dim 128
// and bf16 caches are supported, and cache offsets are 64-bit.
//
// B200 design (one CTA per (split, kv_head, sequence)):
//   - the CTA serves all G = H_q/H_kv query heads of its KV head, so every K/V byte is
//     read from HBM once (the reference re-reads it once per query head);
//   - warp 8 is a producer: it fills a 64 KB shared-memory ring with tiles of ~32 KB (32-128
//     tokens of K and V) found through the block table. When a tile holds whole cache blocks,
//     its lane 0 issues one 3-D TMA load per block for K and one for V (a tensor map over the
//     cache as [P * block_size][H_kv][D]) and the stage barrier counts the bytes; otherwise
//     the warp gathers rows with coalesced 16-byte cp.async and counts completion with
//     cp.async.mbarrier.arrive. 1-D bulk copies of single rows were measured to be
//     request-rate bound here (fp32 and bf16 took equal time);
//   - warps 0..7 consume: each owns a slice of every tile's tokens and runs its own
//     exp2-domain online softmax with no CTA barrier inside the loop; the warps' partial
//     (o, m, l) are merged by log-sum-exp at the end of the split;
//   - 3 CTAs per SM (ring 64 KB) hide the per-CTA start-up and merge latency;
//   - the split merge is fused: every CTA of a (sequence, KV head) writes its partial to
//     the workspace, and the last to arrive (atomic ticket) merges and writes O.
#include "common.cuh"
#include <cuda_bf16.h>
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace b2 {

constexpr int DA_NW = 8;                 // consumer warps
constexpr int DA_NT = (DA_NW + 1) * 32;  // + producer warp
constexpr int DA_MINB = 3;               // CTAs per SM the register budget is sized for (G <= 4)

struct DecodeAttnParams {
    const float* Q;
    const unsigned char* k_cache;
    const unsigned char* v_cache;
    const int* block_table;
    const int* context_lens;
    float* O;
    float* ws_partial;          // [B, H_q, num_splits, D + 2]
    unsigned int* ws_counter;   // [B, H_kv]
    int H_q, H_kv, block_size, num_blocks_per_seq, num_phys_blocks;
    int num_splits, blocks_per_split;
    float scale_log2;           // softmax scale * log2(e)
    unsigned int* err;          // device error word
};

constexpr int ilog2(int x) { return x <= 1 ? 0 : 1 + ilog2(x / 2); }

template <int G, int D, typename KV>
struct DACfg {
    static constexpr int ES = (int)sizeof(KV);
    static constexpr int ROW = D * ES;                 // bytes of one K or V row
    // tokens per tile: about 32 KB of K+V per tile whatever the element size
    static constexpr int T = (16384 / ROW) < 32 ? 32 : ((16384 / ROW) > 128 ? 128 : (16384 / ROW));
    static constexpr int STAGE = 2 * T * ROW;          // K tile then V tile, rows dense
    static constexpr int STAGES_RAW = (64 * 1024) / STAGE;  // 64 KB ring: 3 CTAs per SM
    static constexpr int STAGES = STAGES_RAW < 2 ? 2 : (STAGES_RAW > 8 ? 8 : STAGES_RAW);
    static constexpr int VPL = D / 32;                 // head_dim columns per lane
    static constexpr int TW = T / DA_NW;               // tokens of a tile per consumer warp
    // tokens per consumer group: as many as keep TPW * G <= 16 dot products per reduction
    static constexpr int TPW = (16 / G) < TW ? (16 / G) : TW;
    // shared-memory carve-up (bytes)
    static constexpr int OFF_X = STAGES * STAGE;                         // f32 [NW][32] p / alpha exchange
    static constexpr int OFF_ML = OFF_X + DA_NW * 32 * 4;                // f32 [NW][G][2]
    static constexpr int OFF_BT = OFF_ML + DA_NW * G * 2 * 4;            // i32 [BT_CAP] block-table slice
    static constexpr int BT_CAP = 256;
    static constexpr int OFF_MISC = OFF_BT + BT_CAP * 4;                 // u32 flags
    static constexpr int OFF_BAR = (OFF_MISC + 16 + 7) & ~7;             // u64 full[S], empty[S]
    static constexpr int SMEM = OFF_BAR + 2 * STAGES * 8;
    static_assert(D % 32 == 0, "head_dim must be 64 or 128");
    static_assert(DA_NW * G * D * 4 <= STAGES * STAGE, "final reduction must fit the ring");
    static_assert(TW % TPW == 0 && T % 32 == 0, "tile must split evenly over the consumer warps");
};

// Sum of NV per-lane values across the warp for every index at once: lane l ends with
// the full sum of value (l >> (5 - log2 NV)). Each halving step trades half the values
// with the partner lane, so NV sums cost NV - 1 + (5 - log2 NV) shuffles, not 5 * NV.
template <int NV>
__device__ __forceinline__ float warp_transpose_sum(float (&v)[NV], int lane) {
    constexpr int L = ilog2(NV);
#pragma unroll
    for (int k = 0; k < L; ++k) {
        const int h = NV >> (k + 1);
        const int o = 16 >> k;
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < h; ++i) {
            const float send = up ? v[i] : v[i + h];
            const float keep = up ? v[i + h] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    float r = v[0];
#pragma unroll
    for (int o = 16 >> L; o >= 1; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    return r;
}

// Load N elements of a K/V row from shared memory into fp32 registers.
template <typename KV, int N>
__device__ __forceinline__ void load_row(const unsigned char* p, float (&f)[N]) {
    if constexpr (sizeof(KV) == 4) {
        static_assert(N % 2 == 0, "");
        if constexpr (N % 4 == 0) {
#pragma unroll
            for (int i = 0; i < N / 4; ++i) {
                float4 v = reinterpret_cast<const float4*>(p)[i];
                f[4 * i] = v.x; f[4 * i + 1] = v.y; f[4 * i + 2] = v.z; f[4 * i + 3] = v.w;
            }
        } else {
            float2 v = *reinterpret_cast<const float2*>(p);
            f[0] = v.x; f[1] = v.y;
        }
    } else {
        // bf16 -> fp32 is exact: the bf16 bits are the top half of the fp32 word.
        if constexpr (N % 8 == 0) {
#pragma unroll
            for (int i = 0; i < N / 8; ++i) {
                uint4 v = reinterpret_cast<const uint4*>(p)[i];
                uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    f[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
                    f[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
                }
            }
        } else if constexpr (N == 4) {
            uint2 v = *reinterpret_cast<const uint2*>(p);
            f[0] = __uint_as_float(v.x << 16); f[1] = __uint_as_float(v.x & 0xffff0000u);
            f[2] = __uint_as_float(v.y << 16); f[3] = __uint_as_float(v.y & 0xffff0000u);
        } else {
            static_assert(N == 2, "");
            uint32_t v = *reinterpret_cast<const uint32_t*>(p);
            f[0] = __uint_as_float(v << 16); f[1] = __uint_as_float(v & 0xffff0000u);
        }
    }
}

// ------------------------------------------------------------------ pieces shared by both kernels

// Context length of sequence b, clamped to its block-table row (an overlong length is
// reported once per launch by the caller's choice of `report`).
__device__ __forceinline__ int da_context(const DecodeAttnParams& p, int b, bool report) {
    int ctx = p.context_lens[b];
    const int cap = p.num_blocks_per_seq * p.block_size;
    if (ctx > cap) {
        if (report) raise_error(p.err, B2_DEVERR_CTX_RANGE);
        ctx = cap;
    }
    return ctx < 0 ? 0 : ctx;
}

// Producer warp: gathers tile `i` of the token range [tok_begin, tok_end) of (b, kvh) into
// the stage at sK (K rows) / sV (V rows). Lane r resolves the cache offset of row r of each
// 32-row chunk; the warp then moves rows with coalesced 16-byte cp.async, CPR lanes per row.
// bt_s holds the range's block-table slice when `staged` (else the row is read from global).
template <typename C>
__device__ __forceinline__ void da_issue_tile(const DecodeAttnParams& p, int b, int kvh, int tok_begin, int tok_end,
                                              int i, uint32_t sK, uint32_t sV, const int* bt_s, bool staged,
                                              int lane, uint64_t pol) {
    constexpr int CPR = C::ROW / 16;  // 16-byte chunks per row
    constexpr int RPI = 32 / CPR;     // rows per warp instruction
    constexpr int RC = C::T / 32;     // 32-row chunks per tile
    const int* bt = p.block_table + (size_t)b * p.num_blocks_per_seq;
    const int blk0 = tok_begin / p.block_size;
    auto row_off = [&](int c) -> long long {
        const int t0 = tok_begin + i * C::T + c * 32;
        if (lane >= tok_end - t0) return 0;
        const int pos = t0 + lane;
        const int blk = pos / p.block_size;
        const int slot = pos - blk * p.block_size;
        int phys = staged ? bt_s[blk - blk0] : bt[blk];
        if (p.num_phys_blocks > 0 && (unsigned)phys >= (unsigned)p.num_phys_blocks) {
            raise_error(p.err, B2_DEVERR_BLOCK_RANGE);
            phys = 0;
        }
        return ((((long long)phys * p.block_size + slot) * p.H_kv + kvh) * (long long)C::ROW);
    };
    const int sub = lane / CPR;
    const int chunk = (lane % CPR) * 16;
    const int n = min(C::T, tok_end - (tok_begin + i * C::T));
#pragma unroll
    for (int c = 0; c < RC; ++c) {
        if (c * 32 >= n) break;
        const long long cur = row_off(c);
#pragma unroll 4
        for (int r0 = c * 32; r0 < min(n, c * 32 + 32); r0 += RPI) {
            const int r = r0 + sub;
            const long long off = __shfl_sync(0xffffffffu, cur, r & 31);
            if (r < n) {
                cp_async16(sK + r * C::ROW + chunk, p.k_cache + off + chunk, pol);
                cp_async16(sV + r * C::ROW + chunk, p.v_cache + off + chunk, pol);
            }
        }
    }
}

// One consumer warp's online-softmax state for one (sequence, KV head) work unit. Warp w
// owns tokens [TW w, TW (w+1)) of every tile; lanes span head_dim (VPL columns each), so
// K/V rows are read as contiguous, conflict-free shared loads. The TPW x G dot products of
// a token group are reduced across the warp with a transposed butterfly (about one shuffle
// per dot product), p and alpha are exchanged through warp-private shared memory, and no
// CTA-wide barrier is taken inside the tile loop.
template <int G, int D, typename KV>
struct DAWarp {
    using C = DACfg<G, D, KV>;
    static constexpr int VP = C::VPL / 2;  // q and the accumulator as fp32 pairs (packed f32x2 FMA)
    static constexpr int TPW = C::TPW;     // tokens per group
    static constexpr int NV = TPW * G;     // dot products per group (<= 16)
    static constexpr int SHIFT = 5 - ilog2(NV);
    static constexpr int LG = ilog2(G);
    float2 q[G][VP];
    float2 acc[G][VP];
    float m_run, l_run;  // head my_g; l over this lane's token subset
    int idx, my_t, my_g;
    bool owner;

    __device__ __forceinline__ void begin(const DecodeAttnParams& p, int b, int hq0, int lane) {
        idx = lane >> SHIFT;
        my_t = idx / G;
        my_g = idx % G;
        owner = (lane & ((1 << SHIFT) - 1)) == 0;
        const float* Qb = p.Q + ((size_t)b * p.H_q + hq0) * D;
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int j = 0; j < VP; ++j) {
                q[g][j] = make_float2(Qb[g * D + lane * C::VPL + 2 * j] * p.scale_log2,
                                      Qb[g * D + lane * C::VPL + 2 * j + 1] * p.scale_log2);
                acc[g][j] = make_float2(0.f, 0.f);
            }
        m_run = -INFINITY;
        l_run = 0.f;
    }

    // This warp's token slice of a tile of n tokens (K rows at Kt, V rows at Vt).
    __device__ __forceinline__ void tile(const unsigned char* Kt, const unsigned char* Vt, int n, int warp, int lane,
                                         float* xw) {
#pragma unroll
        for (int grp = 0; grp < C::TW / TPW; ++grp) {
            const int tok0 = warp * C::TW + grp * TPW;
            if (tok0 >= n) break;  // warp-uniform
            float s[NV];
#pragma unroll
            for (int t = 0; t < TPW; ++t) {
                float kf[C::VPL];
                if (tok0 + t < n) {
                    load_row<KV, C::VPL>(Kt + (tok0 + t) * C::ROW + lane * C::VPL * C::ES, kf);
                } else {
#pragma unroll
                    for (int j = 0; j < C::VPL; ++j) kf[j] = 0.f;
                }
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float2 a = make_float2(0.f, 0.f);
#pragma unroll
                    for (int j = 0; j < VP; ++j) a = ffma2(q[g][j], make_float2(kf[2 * j], kf[2 * j + 1]), a);
                    s[t * G + g] = a.x + a.y;
                }
            }
            float sc = warp_transpose_sum<NV>(s, lane);
            if (tok0 + my_t >= n) sc = -INFINITY;
            float tmax = sc;
#pragma unroll
            for (int k = 0; k < ilog2(TPW); ++k)
                tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1 << (SHIFT + LG + k)));
            const float m_new = fmaxf(m_run, tmax);
            const float alpha = m_new == -INFINITY ? 1.f : fast_exp2(m_run - m_new);
            const float pr = sc == -INFINITY ? 0.f : fast_exp2(sc - m_new);
            l_run = fmaf(l_run, alpha, pr);
            m_run = m_new;
            if (owner) {
                xw[idx] = pr;
                if (my_t == 0) xw[16 + my_g] = alpha;
            }
            __syncwarp();
            float al[G], pv[NV];
#pragma unroll
            for (int g = 0; g < G; ++g) al[g] = xw[16 + g];
#pragma unroll
            for (int k = 0; k < NV; ++k) pv[k] = xw[k];
            __syncwarp();
#pragma unroll
            for (int g = 0; g < G; ++g)
#pragma unroll
                for (int j = 0; j < VP; ++j) acc[g][j] = fmul2(acc[g][j], make_float2(al[g], al[g]));
#pragma unroll
            for (int t = 0; t < TPW; ++t) {
                if (tok0 + t < n) {
                    float vf[C::VPL];
                    load_row<KV, C::VPL>(Vt + (tok0 + t) * C::ROW + lane * C::VPL * C::ES, vf);
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float2 pp = make_float2(pv[t * G + g], pv[t * G + g]);
#pragma unroll
                        for (int j = 0; j < VP; ++j)
                            acc[g][j] = ffma2(pp, make_float2(vf[2 * j], vf[2 * j + 1]), acc[g][j]);
                    }
                }
            }
        }
    }

    // l summed over the lanes holding this head's tokens (valid in owner lanes).
    __device__ __forceinline__ float l_total() const {
        float l = owner ? l_run : 0.f;
#pragma unroll
        for (int k = 0; k < ilog2(TPW); ++k) l += __shfl_xor_sync(0xffffffffu, l, 1 << (SHIFT + LG + k));
        return l;
    }
};

// Final stage of a (sequence, KV head) split, by the NC consumer threads: `get(i, o, M, L)`
// gives the split's merged unnormalised output o, max M and sum L for element i = g*D + d.
// One split: O = o / L. Otherwise the split's partial goes to the workspace and the last of
// the nsplit CTAs (or work items) to arrive (atomic ticket) merges all partials into O and
// leaves the counter at zero.
template <int G, int D, int NC, typename Get>
__device__ __forceinline__ void da_finish(const DecodeAttnParams& p, int b, int kvh, int split, int nsplit, int tid,
                                          volatile unsigned int* ticket, Get get) {
    const int hq0 = kvh * G;
    float* O = p.O + ((size_t)b * p.H_q + hq0) * D;
    if (nsplit == 1) {
        for (int i = tid; i < G * D; i += NC) {
            float o, M, L;
            get(i, o, M, L);
            O[i] = L > 0.f ? o / L : 0.f;
        }
        return;
    }
    const size_t rowlen = D + 2;
    for (int i = tid; i < G * D; i += NC) {
        const int g = i / D, d = i - g * D;
        float o, M, L;
        get(i, o, M, L);
        float* ws = p.ws_partial + (((size_t)b * p.H_q + hq0 + g) * p.num_splits + split) * rowlen;
        ws[d] = o;
        if (d == 0) { ws[D] = M; ws[D + 1] = L; }
    }
    __threadfence();
    named_barrier(1, NC);
    unsigned int* counter = p.ws_counter + (size_t)b * p.H_kv + kvh;
    if (tid == 0) *ticket = atomicAdd(counter, 1u);
    named_barrier(1, NC);
    if (*ticket != (unsigned)(nsplit - 1)) return;
    __threadfence();
    for (int i = tid; i < G * D; i += NC) {
        const int g = i / D, d = i - g * D;
        const float* ws = p.ws_partial + ((size_t)b * p.H_q + hq0 + g) * p.num_splits * rowlen;
        float M = -INFINITY;
        for (int s = 0; s < nsplit; ++s) M = fmaxf(M, __ldcg(ws + s * rowlen + D));
        float L = 0.f, o = 0.f;
        for (int s = 0; s < nsplit; ++s) {
            const float w = fast_exp2(__ldcg(ws + s * rowlen + D) - M);
            L = fmaf(__ldcg(ws + s * rowlen + D + 1), w, L);
            o = fmaf(__ldcg(ws + s * rowlen + d), w, o);
        }
        O[i] = L > 0.f ? o / L : 0.f;
    }
    if (tid == 0) *counter = 0u;  // every sibling has arrived: leave the counter reusable
}

// ------------------------------------------------------------------ the kernel
// Grid (KV head, split, sequence): the CTA's warps merge through the ring's memory once the
// producer is done.
// TMA = true: the producer's lane 0 moves each cache block of the tile with two 3-D TMA loads
// (box head_dim x 1 head x block_size tokens of a tensor map over [P * block_size, H_kv,
// head_dim]) into the same dense rows, completion counted in bytes on the stage's barrier;
// used when tiles hold whole blocks and the pool size is known. Otherwise the warp gathers
// rows with cp.async.
template <int G, int D, typename KV, bool TMA>
__global__ void __launch_bounds__(DA_NT, G >= 8 ? 2 : DA_MINB)
decode_attn_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                   const DecodeAttnParams p) {
    using C = DACfg<G, D, KV>;
    extern __shared__ __align__(1024) unsigned char smem[];
    // KV head fastest in the grid: the CTAs of one token range run side by side
    const int kvh = blockIdx.x;
    const int split = blockIdx.y;
    const int b = blockIdx.z;
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;

    griddep_wait();
    griddep_launch();
    // ---- this CTA's token range (whole blocks, as the reference splits, 13_decode_attn.cu:63-65)
    const int ctx = da_context(p, b, tid == 0 && split == 0 && kvh == 0);
    const int nblk = (ctx + p.block_size - 1) / p.block_size;
    const int nsplit = (nblk + p.blocks_per_split - 1) / p.blocks_per_split;  // non-empty splits
    const int hq0 = kvh * G;

    if (nblk == 0) {  // empty context: O = 0 (reference reduce writes o * 0, 13_decode_attn.cu:48-52)
        float* O = p.O + ((size_t)b * p.H_q + hq0) * D;
        if (split == 0)
            for (int i = tid; i < G * D; i += DA_NT) O[i] = 0.f;
        return;
    }
    if (split >= nsplit) return;  // empty split: contributes nothing

    const int tok_begin = split * p.blocks_per_split * p.block_size;
    const int tok_end = min(ctx, (split + 1) * p.blocks_per_split * p.block_size);
    const int ntiles = (tok_end - tok_begin + C::T - 1) / C::T;

    volatile unsigned int* misc = reinterpret_cast<volatile unsigned int*>(smem + C::OFF_MISC);
    const uint32_t bar0 = smem_u32(smem + C::OFF_BAR);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (C::STAGES + s); };
    const uint32_t ring = smem_u32(smem);

    if (tid == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(full_bar(s), TMA ? 1 : 32);  // TMA: lane 0's expect_tx; else one cp.async arrival per lane
            mbar_init(empty_bar(s), DA_NW);
        }
        misc[0] = 0;  // abort flag
        misc[1] = 0;  // merge ticket
        fence_mbar_init();
    }
    __syncthreads();

    if constexpr (TMA) {
        if (warp == DA_NW) {
            // the split's slice of the block table in shared memory (all lanes), then lane 0
            // issues the copies
            const int* btg = p.block_table + (size_t)b * p.num_blocks_per_seq;
            const int blk0 = tok_begin / p.block_size;
            const int nbt = (tok_end - 1) / p.block_size - blk0 + 1;
            int* bt_s = reinterpret_cast<int*>(smem + C::OFF_BT);
            const bool staged = nbt <= C::BT_CAP;
            if (staged) {
                for (int j = lane; j < nbt; j += 32) bt_s[j] = btg[blk0 + j];
                __syncwarp();
            }
            if (lane == 0) {
                prefetch_tensormap(&kmap);
                prefetch_tensormap(&vmap);
                const uint64_t pol = policy_evict_first();
                const int bs = p.block_size;
                const uint32_t block_bytes = (uint32_t)(bs * C::ROW);
                int issued = 0;  // tiles whose copies were all requested
                for (int i = 0; i < ntiles; ++i) {
                    const int st = i % C::STAGES;
                    if (i >= C::STAGES &&
                        (misc[0] != 0 || !mbar_wait(empty_bar(st), ((i / C::STAGES) - 1) & 1, p.err))) {
                        misc[0] = 1;
                        break;
                    }
                    const int t0 = tok_begin + i * C::T;
                    const int n = min(C::T, tok_end - t0);
                    const int nb = (n + bs - 1) / bs;  // whole blocks (the last may run past the context)
                    const uint32_t sK = ring + st * C::STAGE;
                    mbar_arrive_expect_tx(full_bar(st), 2u * nb * block_bytes);
                    for (int j = 0; j < nb; ++j) {
                        int phys = staged ? bt_s[t0 / bs + j - blk0] : btg[t0 / bs + j];
                        if ((unsigned)phys >= (unsigned)p.num_phys_blocks) {
                            raise_error(p.err, B2_DEVERR_BLOCK_RANGE);
                            phys = 0;
                        }
                        tma_load_3d(sK + j * block_bytes, &kmap, 0, kvh, phys * bs, full_bar(st), pol);
                        tma_load_3d(sK + C::T * C::ROW + j * block_bytes, &vmap, 0, kvh, phys * bs, full_bar(st), pol);
                    }
                    issued = i + 1;
                }
                // drain: the last fill of every stage this thread requested has landed before
                // the CTA can exit, also when a consumer gave up waiting on one
                for (int j = max(0, issued - C::STAGES); j < issued; ++j)
                    mbar_wait_drain(full_bar(j % C::STAGES), (j / C::STAGES) & 1);
            }
            return;
        }
    }
    if (warp == DA_NW) {
        // ------------------------------------------------------------ producer warp
        // The split's slice of the block table is staged in shared memory once, so no tile
        // waits on a dependent global load (long splits fall back to global reads); every lane
        // arrives on the stage's full barrier once its copies have landed.
        const int* bt = p.block_table + (size_t)b * p.num_blocks_per_seq;
        const int blk0 = tok_begin / p.block_size;
        const int nbt = (tok_end - 1) / p.block_size - blk0 + 1;
        int* bt_s = reinterpret_cast<int*>(smem + C::OFF_BT);
        const bool staged = nbt <= C::BT_CAP;
        if (staged) {
            for (int j = lane; j < nbt; j += 32) bt_s[j] = bt[blk0 + j];
            __syncwarp();
        }
        const uint64_t pol = policy_evict_first();
        for (int i = 0; i < ntiles; ++i) {
            const int st = i % C::STAGES;
            if (i >= C::STAGES) {
                const uint32_t par = ((i / C::STAGES) - 1) & 1;
                bool ok = misc[0] == 0 && mbar_wait(empty_bar(st), par, p.err);
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                if (!ok) { if (lane == 0) misc[0] = 1; break; }
            }
            const uint32_t sK = ring + st * C::STAGE;
            da_issue_tile<C>(p, b, kvh, tok_begin, tok_end, i, sK, sK + C::T * C::ROW, bt_s, staged, lane, pol);
            cp_async_mbar_arrive_noinc(full_bar(st));
        }
        cp_async_wait_all();  // nothing may still be landing in the ring when the warp exits
        return;
    }

    // ---------------------------------------------------------------- consumer warps
    constexpr int NC = DA_NW * 32;
    float* xw = reinterpret_cast<float*>(smem + C::OFF_X) + warp * 32;  // [0,NV) p, [16,16+G) alpha
    DAWarp<G, D, KV> w;
    w.begin(p, b, hq0, lane);
    for (int i = 0; i < ntiles; ++i) {
        const int st = i % C::STAGES;
        const int n = min(C::T, tok_end - (tok_begin + i * C::T));
        if (misc[0] == 0) {
            if (!mbar_wait(full_bar(st), (i / C::STAGES) & 1, p.err)) misc[0] = 1;
        }
        const unsigned char* Kt = smem + st * C::STAGE;
        w.tile(Kt, Kt + C::T * C::ROW, n, warp, lane, xw);
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(st));
    }

    // ---- merge the 8 warps through the ring's memory (the producer is done with it)
    const float l_tot = w.l_total();
    named_barrier(1, NC);  // every warp is done reading the ring
    float* red = reinterpret_cast<float*>(smem);               // [NW][G][D]
    float* ml_s = reinterpret_cast<float*>(smem + C::OFF_ML);  // [NW][G][2]
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < DAWarp<G, D, KV>::VP; ++j) {
            red[(warp * G + g) * D + lane * C::VPL + 2 * j] = w.acc[g][j].x;
            red[(warp * G + g) * D + lane * C::VPL + 2 * j + 1] = w.acc[g][j].y;
        }
    if (w.owner && w.my_t == 0) {
        ml_s[(warp * G + w.my_g) * 2] = w.m_run;
        ml_s[(warp * G + w.my_g) * 2 + 1] = l_tot;
    }
    named_barrier(1, NC);
    if (misc[0] != 0) return;  // a wait gave up: the error bit is set, O is left untouched
    // log-sum-exp merge of the 8 warps for element i = g*D + d -> (o, M, L)
    auto merge_warps = [&](int i, float& o, float& M, float& L) {
        const int g = i / D;
        M = -INFINITY;
#pragma unroll
        for (int v = 0; v < DA_NW; ++v) M = fmaxf(M, ml_s[(v * G + g) * 2]);
        o = 0.f;
        L = 0.f;
        if (M == -INFINITY) return;
#pragma unroll
        for (int v = 0; v < DA_NW; ++v) {
            const float mw = ml_s[(v * G + g) * 2];
            if (mw == -INFINITY) continue;
            const float sc = fast_exp2(mw - M);
            o = fmaf(red[v * G * D + i], sc, o);
            L = fmaf(ml_s[(v * G + g) * 2 + 1], sc, L);
        }
    };
    da_finish<G, D, NC>(p, b, kvh, split, nsplit, tid, misc + 1, merge_warps);
}

// ------------------------------------------------------------------ host side

struct SplitPlan {
    int num_splits;
    int blocks_per_split;
};

// Split policy: enough CTAs to fill the GPU a few times over, and no CTA streaming more
// than ~512 KB of K+V, so ragged batches balance; capped by max_splits and by a floor of
// 64 tokens per split. When the
// (sequence, KV head) pairs cannot fill the SMs (a shard of the heads on one of several
// GPUs), CTAs shrink (down to 256 tokens) so that the upper bound B * H_kv * max_ctx of the
// work spans ~4 waves of 3 CTAs per SM.
static SplitPlan plan_splits(int B, int H_kv, int head_dim, int kv_bytes, int max_ctx, int block_size,
                             int max_splits, int num_sms) {
    const int max_blocks = std::max(1, (max_ctx + block_size - 1) / block_size);
    const long long pairs = (long long)B * H_kv;
    const long long row_bytes = 2LL * head_dim * kv_bytes;           // K + V bytes per token
    const long long cap_tok = (512LL * 1024) / row_bytes;
    const long long waves_tok = pairs * max_ctx / (4LL * DA_MINB * num_sms);
    const long long tok_per_cta =
        pairs >= num_sms ? std::max<long long>(64, cap_tok)
                         : std::max<long long>(256, std::min<long long>(waves_tok, cap_tok));
    long long want = std::max<long long>((4LL * num_sms + pairs - 1) / pairs,
                                         ((long long)max_ctx + tok_per_cta - 1) / tok_per_cta);
    // at least 2 blocks and 64 tokens of work per split: below that a CTA's fixed start-up
    // and the wider merge cost more than the parallelism gains (config 1, B1 H12 ctx 1024:
    // 32 splits 8.2 us, 16 splits 7.2 us, 8 splits 7.1 us, 4 splits 8.9 us)
    want = std::min<long long>(want, std::max(1, max_blocks / 2));
    want = std::min<long long>(want, std::max(1, (max_ctx + 63) / 64));
    want = std::max<long long>(1, std::min<long long>(want, max_splits));
    SplitPlan sp;
    sp.blocks_per_split = (int)((max_blocks + want - 1) / want);
    sp.num_splits = (max_blocks + sp.blocks_per_split - 1) / sp.blocks_per_split;
    return sp;
}

bool set_smem_attr_once(const void* func, int bytes, int slot);

int num_sms_current_device();

typedef CUresult (*DaEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Tensor map over a K or V cache [P, block_size, H_kv, D] as [P * block_size][H_kv][D] with a
// box of D x 1 x block_size (one head of one block); cached per (device, pointer, shape).
template <typename KV>
static bool kv_map(CUtensorMap* map, const void* cache, long long tokens, int H_kv, int D, int block_size) {
    struct Entry { int dev; const void* base; long long tokens; int H, D, bs; CUtensorMap map; };
    constexpr int kEntries = 64;
    static Entry cache_[kEntries];
    static int fill = 0, next = 0;
    static std::mutex mu;
    static DaEncodeFn enc = nullptr;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    for (int i = 0; i < fill; ++i) {
        const Entry& e = cache_[i];
        if (e.dev == dev && e.base == cache && e.tokens == tokens && e.H == H_kv && e.D == D && e.bs == block_size) {
            *map = e.map;
            return true;
        }
    }
    if (!enc) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return false;
        enc = reinterpret_cast<DaEncodeFn>(ptr);
    }
    const cuuint64_t es = sizeof(KV);
    cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)H_kv, (cuuint64_t)tokens};
    cuuint64_t strides[2] = {(cuuint64_t)D * es, (cuuint64_t)H_kv * D * es};
    cuuint32_t box[3] = {(cuuint32_t)D, 1, (cuuint32_t)block_size};
    cuuint32_t estr[3] = {1, 1, 1};
    if (enc(map, sizeof(KV) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
            const_cast<void*>(cache), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
        return false;
    Entry& e = cache_[next];
    e = Entry{dev, cache, tokens, H_kv, D, block_size, *map};
    next = (next + 1) % kEntries;
    if (fill < kEntries) ++fill;
    return true;
}

template <int G, int D, typename KV>
static cudaError_t launch_decode_attn_t(const DecodeAttnParams& prm, int B, cudaStream_t st) {
    using C = DACfg<G, D, KV>;
    dim3 grid(prm.H_kv, prm.num_splits, B);
    CUtensorMap km, vm;
    static const bool tma_off = getenv("B2_ATTN_TMA") && strcmp(getenv("B2_ATTN_TMA"), "0") == 0;
    const bool tma = !tma_off && prm.num_phys_blocks > 0 && prm.block_size <= 256 && C::T % prm.block_size == 0 &&
                     kv_map<KV>(&km, prm.k_cache, (long long)prm.num_phys_blocks * prm.block_size, prm.H_kv, D,
                                prm.block_size) &&
                     kv_map<KV>(&vm, prm.v_cache, (long long)prm.num_phys_blocks * prm.block_size, prm.H_kv, D,
                                prm.block_size);
    if (tma) {
        if (!set_smem_attr_once((const void*)decode_attn_kernel<G, D, KV, true>, C::SMEM, 0)) return cudaErrorInvalidValue;
        return launch_kernel(decode_attn_kernel<G, D, KV, true>, grid, dim3(DA_NT), (size_t)C::SMEM, st, km, vm, prm);
    }
    memset(&km, 0, sizeof(km));
    if (!set_smem_attr_once((const void*)decode_attn_kernel<G, D, KV, false>, C::SMEM, 0)) return cudaErrorInvalidValue;
    return launch_kernel(decode_attn_kernel<G, D, KV, false>, grid, dim3(DA_NT), (size_t)C::SMEM, st, km, km, prm);
}

template <int D, typename KV>
static cudaError_t dispatch_group(int G, const DecodeAttnParams& prm, int B, cudaStream_t st) {
    switch (G) {
        case 1: return launch_decode_attn_t<1, D, KV>(prm, B, st);
        case 2: return launch_decode_attn_t<2, D, KV>(prm, B, st);
        case 4: return launch_decode_attn_t<4, D, KV>(prm, B, st);
        case 8: return launch_decode_attn_t<8, D, KV>(prm, B, st);
        default: return cudaErrorInvalidValue;
    }
}

// Workspace layout: [B, H_q, num_splits, D+2] f32 partials, then [B, H_kv] u32 counters
// (256-byte aligned).
static size_t partial_bytes(int B, int H_q, int D, int S) {
    size_t b = (size_t)B * H_q * S * (D + 2) * sizeof(float);
    return (b + 255) & ~(size_t)255;
}


// Largest split count whose workspace fits the allocation-free entry point's fixed array
// (1 when not even two splits fit: a single split needs no workspace).
int noalloc_max_splits(int B, int H_q, int H_kv, int D) {
    if (B <= 0 || H_q <= 0 || H_kv <= 0 || D <= 0) return 1;
    const size_t counters = (size_t)B * H_kv * sizeof(unsigned int);
    int s = 64;
    while (s > 1 && partial_bytes(B, H_q, D, s) + counters > (size_t)B2_DECODE_NOALLOC_SCRATCH_BYTES) --s;
    return s;
}

size_t decode_attn_workspace_size(int B, int H_q, int H_kv, int D, int max_ctx, int block_size,
                                  int max_splits, int kv_bytes) {
    SplitPlan sp = plan_splits(B, H_kv, D, kv_bytes, max_ctx, block_size, max_splits, num_sms_current_device());
    return partial_bytes(B, H_q, D, sp.num_splits) + (size_t)B * H_kv * sizeof(unsigned int);
}

// Validates, plans and launches. `max_splits` bounds the split count (the drop-in
// wrapper passes the reference workspace's capacity). `counters_zeroed` false makes the
// launcher clear the counter region first (stream-ordered memset).
int decode_attn_launch(const b2_decode_attn_args* a, int max_splits, bool counters_zeroed, cudaStream_t st) {
    if (!a) return B2_ERR_INVALID;
    if (a->B < 0 || a->H_q <= 0 || a->H_kv <= 0 || a->block_size <= 0 || a->num_blocks_per_seq < 0 ||
        a->max_context_len < 0)
        return B2_ERR_INVALID;
    if (a->B == 0) return B2_OK;
    if (!a->Q || !a->k_cache || !a->v_cache || !a->block_table || !a->context_lens || !a->O)
        return B2_ERR_INVALID;
    if (a->H_q % a->H_kv != 0) return B2_ERR_UNSUPPORTED;
    const int G = a->H_q / a->H_kv;
    if (G != 1 && G != 2 && G != 4 && G != 8) return B2_ERR_UNSUPPORTED;
    if (a->head_dim != 64 && a->head_dim != 128) return B2_ERR_UNSUPPORTED;
    if (a->kv_dtype != B2_KV_F32 && a->kv_dtype != B2_KV_BF16) return B2_ERR_UNSUPPORTED;
    if (((uintptr_t)a->k_cache | (uintptr_t)a->v_cache) & 15) return B2_ERR_INVALID;  // bulk-copy alignment
    if (((uintptr_t)a->Q | (uintptr_t)a->O) & 15) return B2_ERR_INVALID;
    const int kvb = a->kv_dtype == B2_KV_F32 ? 4 : 2;

    SplitPlan sp = plan_splits(a->B, a->H_kv, a->head_dim, kvb, a->max_context_len, a->block_size, max_splits,
                               num_sms_current_device());
    DecodeAttnParams prm;
    prm.Q = a->Q;
    prm.k_cache = static_cast<const unsigned char*>(a->k_cache);
    prm.v_cache = static_cast<const unsigned char*>(a->v_cache);
    prm.block_table = a->block_table;
    prm.context_lens = a->context_lens;
    prm.O = a->O;
    prm.H_q = a->H_q;
    prm.H_kv = a->H_kv;
    prm.block_size = a->block_size;
    prm.num_blocks_per_seq = a->num_blocks_per_seq;
    prm.num_phys_blocks = a->num_phys_blocks;
    prm.num_splits = sp.num_splits;
    prm.blocks_per_split = sp.blocks_per_split;
    const float scale = a->scale != 0.f ? a->scale : 1.0f / sqrtf((float)a->head_dim);
    prm.scale_log2 = scale * 1.4426950408889634f;
    prm.err = device_error_ptr();
    prm.ws_partial = nullptr;
    prm.ws_counter = nullptr;
    if (sp.num_splits > 1) {
        const size_t pb = partial_bytes(a->B, a->H_q, a->head_dim, sp.num_splits);
        const size_t need = pb + (size_t)a->B * a->H_kv * sizeof(unsigned int);
        if (!a->workspace || a->workspace_bytes < need) return B2_ERR_WORKSPACE;
        if ((uintptr_t)a->workspace & 255) return B2_ERR_INVALID;
        prm.ws_partial = static_cast<float*>(a->workspace);
        prm.ws_counter = reinterpret_cast<unsigned int*>(static_cast<char*>(a->workspace) + pb);
        if (!counters_zeroed) {
            if (cudaMemsetAsync(prm.ws_counter, 0, (size_t)a->B * a->H_kv * sizeof(unsigned int), st) !=
                cudaSuccess)
                return B2_ERR_CUDA;
        }
    }
    cudaError_t e;
    if (a->head_dim == 64)
        e = kvb == 4 ? dispatch_group<64, float>(G, prm, a->B, st) : dispatch_group<64, __nv_bfloat16>(G, prm, a->B, st);
    else
        e = kvb == 4 ? dispatch_group<128, float>(G, prm, a->B, st) : dispatch_group<128, __nv_bfloat16>(G, prm, a->B, st);
    return e == cudaSuccess ? B2_OK : B2_ERR_CUDA;
}

}  // namespace b2

// ------------------------------------------------------------------ allocation-free variant
// For callers that cannot call cudaMalloc (see b2_decode_attn_noalloc in b2decode.h): the
// split workspace lives in this fixed device array instead of caller memory. Every GPU that
// loads the library holds it until the process exits. Host code must not pass the array's
// name to a kernel — on the host it is only a stand-in symbol — so its device address is
// looked up once per device with cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_decode_noalloc_scratch[B2_DECODE_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kNoAllocMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (first call per device does
// the lookup; returns nullptr on failure).
void* noalloc_scratch_address() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_decode_noalloc_scratch) != cudaSuccess) return nullptr;
        g_noalloc_addr[dev] = p;
    }
    return g_noalloc_addr[dev];
}
}  // namespace

extern "C" int b2_decode_attn_noalloc(const b2_decode_attn_args* args, b2_stream_t stream) {
    if (!args) return B2_ERR_INVALID;
    void* scratch = noalloc_scratch_address();
    if (!scratch) return B2_ERR_CUDA;
    b2_decode_attn_args a = *args;
    a.workspace = scratch;
    a.workspace_bytes = B2_DECODE_NOALLOC_SCRATCH_BYTES;
    // The split count is capped by what the fixed array holds: the largest S whose partials
    // [B, H_q, S, d+2] plus the [B, H_kv] counters fit, at most b2_decode_attn's cap of 64.
    // A plan with one split uses no scratch, so no shape is refused for its size; large
    // batches simply run with fewer splits. The arrival counters are cleared with a
    // stream-ordered memset on every call, since the array keeps whatever the previous
    // call left in it.
    return b2::decode_attn_launch(&a, b2::noalloc_max_splits(a.B, a.H_q, a.H_kv, a.head_dim),
                                  false, static_cast<cudaStream_t>(stream));
}
