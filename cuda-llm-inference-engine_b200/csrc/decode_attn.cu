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
// B200 design:
//   - work schedule: every CTA of one wave reads the context lengths and streams an equal
//     share of the batch's cache blocks (units = (sequence, KV head) laid end to end, each
//     charged a start-and-merge cost), so ragged batches balance; a unit cut across CTAs is
//     merged from its pieces. Short units that fill the GPU by themselves run whole, two per
//     CTA (decode_attn_pair_kernel) for head_dim 64;
//   - the CTA serves all G = H_q/H_kv query heads of its KV head, so every K/V byte is
//     read from HBM once (the reference re-reads it once per query head);
//   - warp 8 is a producer: it fills a 64 KB (96 KB for G 4 / d 128) shared-memory ring with
//     tiles of ~32 KB (32-128 tokens of K and V) found through the block table. When a tile
//     holds whole cache blocks, its lane 0 issues one 3-D TMA load per block for K and one for
//     V (a tensor map over the cache as [P * block_size][H_kv][D]) and the stage barrier counts
//     the bytes; otherwise the warp gathers rows with coalesced 16-byte cp.async and counts
//     completion with cp.async.mbarrier.arrive. 1-D bulk copies of single rows were measured
//     to be request-rate bound here (fp32 and bf16 took equal time);
//   - warps 0..7 consume: each owns a slice of every tile's tokens and runs its own
//     exp2-domain online softmax with no CTA barrier inside the loop; the warps' partial
//     (o, m, l) are merged by log-sum-exp at the end of each unit's piece;
//   - 3 CTAs per SM (2 for G 4 / d 128 and G 8) hide the per-CTA start-up and merge latency;
//   - the split merge is fused: every piece of a cut unit goes to the workspace, and the
//     last to arrive (atomic ticket) merges them and writes O.
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
constexpr int DA_XW = 48;                // floats per warp of the p / alpha exchange (alpha at 32)
// G = 4, head_dim 128: 2 CTAs per SM with a 96 KB ring and token groups of
// 8 (32 dot products per reduction) instead of 3 CTAs with 64 KB and groups of 4: the registers
// of 2 CTAs per SM hold the wider groups without spilling, and each SM keeps 192 KB in flight.
// Config 3: fp32 187 -> 182 us, bf16 131 -> 116 us, the 8-way head shard 34.8 -> 31.5 us.
template <int G, int D, typename KV>
constexpr bool da_wide() { return G == 4 && D == 128; }
template <int G, int D, typename KV>
constexpr int da_minb() { return G >= 8 ? 2 : (da_wide<G, D, KV>() ? 2 : DA_MINB); }

constexpr int DA_MAX_B = 256;           // sequences per launch of the kernel (larger batches are chunked)

struct DecodeAttnParams {
    const float* Q;
    const unsigned char* k_cache;
    const unsigned char* v_cache;
    const int* block_table;
    const int* context_lens;
    float* O;
    float* ws_partial;          // [pieces][G][D + 2] partial (o, m, l) of every piece of a unit
    unsigned int* ws_counter;   // [B * H_kv] arrival tickets
    int B;                      // sequences of this launch (<= DA_MAX_B)
    int H_q, H_kv, block_size, num_blocks_per_seq, num_phys_blocks;
    int chunk_min;              // fewest cache blocks a CTA streams (balanced plan)
    int unit_cost;              // blocks' worth of time a CTA spends starting and merging a unit
    // decode engine, two-units-per-CTA kernel: the caches' blocks before each sequence's last
    // one, the block table and the context lengths were written before the previous kernel on
    // the stream, so they are read before waiting on it (only Q and the newest token's block
    // wait); the public entry points leave this 0 and read nothing before the wait
    int kv_early;
    int unit_mode;              // 1: CTA u serves (sequence, KV head) unit u whole, no workspace
    float scale_log2;           // softmax scale * log2(e)
    unsigned int* err;          // device error word
};

constexpr int ilog2(int x) { return x <= 1 ? 0 : 1 + ilog2(x / 2); }

// GR: independent warp groups per CTA, each streaming its own unit through its own half of
// the ring (GR = 2 for short units: two units per CTA, so a GPT-2 layer's 768 units fit in
// one wave of 3 CTAs per SM).
template <int G, int D, typename KV, int GR = 1>
struct DACfg {
    static constexpr int ES = (int)sizeof(KV);
    static constexpr int ROW = D * ES;                 // bytes of one K or V row
    static constexpr int NWG = DA_NW / GR;             // consumer warps per group
    // tokens per tile: about 32 KB of K+V per tile (per CTA) whatever the element size
    static constexpr int T1 = (16384 / ROW) < 32 ? 32 : ((16384 / ROW) > 128 ? 128 : (16384 / ROW));
    static constexpr int T = T1 / GR;
    static constexpr int STAGE = 2 * T * ROW;          // K tile then V tile, rows dense
    // 64 KB ring: 3 CTAs per SM (96 KB, 2 CTAs per SM, for da_wide)
    static constexpr int RING = da_wide<G, D, KV>() ? 96 * 1024 : 64 * 1024;
    static constexpr int STAGES_RAW = RING / (GR * STAGE);
    static constexpr int STAGES = STAGES_RAW < 2 ? 2 : (STAGES_RAW > 8 ? 8 : STAGES_RAW);
    static constexpr int VPL = D / 32;                 // head_dim columns per lane
    static constexpr int TW = T / NWG;                 // tokens of a tile per consumer warp
    // tokens per consumer group: as many as keep TPW * G <= 16 dot products per reduction
    static constexpr int NVMAX = da_wide<G, D, KV>() ? 32 : 16;
    static constexpr int TPW = (NVMAX / G) < TW ? (NVMAX / G) : TW;
    // shared-memory carve-up (bytes)
    static constexpr int OFF_X = GR * STAGES * STAGE;                    // f32 [NW][32] p / alpha exchange
    static constexpr int OFF_ML = OFF_X + DA_NW * DA_XW * 4;             // f32 [NW][G][2]
    static constexpr int OFF_BT = OFF_ML + DA_NW * G * 2 * 4;            // i32 [BT_CAP] block-table slice
    static constexpr int BT_CAP = 256;                                   // (BT_CAP / GR per group)
    static constexpr int OFF_P = OFF_BT + BT_CAP * 4;                    // i32 [DA_MAX_B + 1] block prefix
    static constexpr int OFF_CTX = OFF_P + (DA_MAX_B + 4) * 4;           // i32 [DA_MAX_B] context lengths
    static constexpr int OFF_MISC = OFF_CTX + DA_MAX_B * 4;              // u32 flags
    static constexpr int OFF_BAR = (OFF_MISC + 16 + 7) & ~7;             // u64 full[GR][S], empty[GR][S]
    static constexpr int SMEM = OFF_BAR + 2 * GR * STAGES * 8;
    static_assert(D % 32 == 0, "head_dim must be 64 or 128");
    static_assert(NWG * G * D * 4 <= STAGE, "the warps' merge must fit one ring stage");
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
template <int G, int D, typename KV, int GR = 1>
struct DAWarp {
    using C = DACfg<G, D, KV, GR>;
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
    // A full tile (n == T, most of them) takes a copy of the loop with every token bound
    // known at compile time, so it carries no per-token range checks.
    __device__ __forceinline__ void tile(const unsigned char* Kt, const unsigned char* Vt, int n, int warp, int lane,
                                         float* xw) {
        if (n == C::T)
            tile_n<true>(Kt, Vt, C::T, warp, lane, xw);
        else
            tile_n<false>(Kt, Vt, n, warp, lane, xw);
    }

    template <bool FULL>
    __device__ __forceinline__ void tile_n(const unsigned char* Kt, const unsigned char* Vt, int n, int warp, int lane,
                                           float* xw) {
        if constexpr (FULL) n = C::T;
#pragma unroll
        for (int grp = 0; grp < C::TW / TPW; ++grp) {
            const int tok0 = warp * C::TW + grp * TPW;
            if (!FULL && tok0 >= n) break;  // warp-uniform
            float s[NV];
#pragma unroll
            for (int t = 0; t < TPW; ++t) {
                float kf[C::VPL];
                if (FULL || tok0 + t < n) {
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
            if (!FULL && tok0 + my_t >= n) sc = -INFINITY;
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
                if (my_t == 0) xw[32 + my_g] = alpha;
            }
            __syncwarp();
            float al[G], pv[NV];
#pragma unroll
            for (int g = 0; g < G; ++g) al[g] = xw[32 + g];
#pragma unroll
            for (int k = 0; k < NV; ++k) pv[k] = xw[k];
            __syncwarp();
#pragma unroll
            for (int g = 0; g < G; ++g)
#pragma unroll
                for (int j = 0; j < VP; ++j) acc[g][j] = fmul2(acc[g][j], make_float2(al[g], al[g]));
#pragma unroll
            for (int t = 0; t < TPW; ++t) {
                if (FULL || tok0 + t < n) {
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

// Floats of one piece in the workspace: o [G][D], then (M, L) [G][2] padded to 16 bytes, so
// every piece and every head's o row starts 16-byte aligned.
template <int G, int D>
constexpr int da_piece_floats() { return G * D + ((2 * G + 3) & ~3); }

// Final stage of a piece of a (sequence, KV head) unit, by the NC consumer threads:
// `get(i, o, M, L)` gives the piece's merged unnormalised output o, max M and sum L for
// element i = g*D + d. A unit in one piece: O = o / L. Otherwise the piece goes to workspace
// row `slot0 + split` and the last of the unit's nsplit pieces to arrive (atomic ticket on
// the unit's counter) merges all of them into O and leaves the counter at zero. `scratch`
// (shared memory, >= 2 * nsplit * G + 4 * NC floats) may alias what `get` reads.
template <int G, int D, int NC, typename Get>
__device__ __forceinline__ void da_finish(const DecodeAttnParams& p, int b, int kvh, int split, int nsplit,
                                          int slot0, int tid, volatile unsigned int* ticket, float* scratch,
                                          Get get) {
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
    constexpr int piece = da_piece_floats<G, D>();
    float* ws0 = p.ws_partial + (size_t)slot0 * piece;
    {
        float* ws = ws0 + (size_t)split * piece;
        for (int i = tid; i < G * D; i += NC) {
            float o, M, L;
            get(i, o, M, L);
            ws[i] = o;
            if ((i & (D - 1)) == 0) {
                ws[G * D + 2 * (i / D)] = M;
                ws[G * D + 2 * (i / D) + 1] = L;
            }
        }
    }
    __threadfence();
    named_barrier(1, NC);
    unsigned int* counter = p.ws_counter + (size_t)b * p.H_kv + kvh;
    if (tid == 0) *ticket = atomicAdd(counter, 1u);
    named_barrier(1, NC);
    const bool last = *ticket == (unsigned)(nsplit - 1);
    named_barrier(1, NC);  // every thread has read the ticket (and is done with `get`)
    if (!last) return;
    __threadfence();
    // (M, L) of every piece into shared memory in one round of independent loads
    float* Ms = scratch;               // [nsplit][G]
    float* Ls = scratch + nsplit * G;  // [nsplit][G]
    for (int j = tid; j < nsplit * G; j += NC) {
        const int sp = j / G, g = j - sp * G;
        const float* ml = ws0 + (size_t)sp * piece + G * D + 2 * g;
        Ms[j] = __ldcg(ml);
        Ls[j] = __ldcg(ml + 1);
    }
    named_barrier(1, NC);
    // Outputs in groups of 4 (NQ of them); the NC threads form SG piece groups, thread
    // (sg, i4) summing pieces sg, sg + SG, ... of group i4 with 16-byte loads, so the loads of
    // all pieces are in flight together; the SG partial sums then meet in shared memory.
    constexpr int NQ = G * D / 4;
    constexpr int SG = NC / NQ > 0 ? NC / NQ : 1;
    float4* part = reinterpret_cast<float4*>(scratch + ((2 * nsplit * G + 3) & ~3));  // [SG][NQ]
    for (int j = tid; j < SG * NQ; j += NC) {
        const int sg = j / NQ, i4 = j - sg * NQ;
        const int g = (i4 * 4) / D;
        float M = -INFINITY;
        for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, Ms[sp * G + g]);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (int sp = sg; sp < nsplit; sp += SG) {
            const float w = fast_exp2(Ms[sp * G + g] - M);
            const float4 v = __ldcg(reinterpret_cast<const float4*>(ws0 + (size_t)sp * piece) + i4);
            acc.x = fmaf(v.x, w, acc.x);
            acc.y = fmaf(v.y, w, acc.y);
            acc.z = fmaf(v.z, w, acc.z);
            acc.w = fmaf(v.w, w, acc.w);
        }
        part[j] = acc;
    }
    named_barrier(1, NC);
    for (int i4 = tid; i4 < NQ; i4 += NC) {
        const int g = (i4 * 4) / D;
        float M = -INFINITY;
        for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, Ms[sp * G + g]);
        float L = 0.f;
        for (int sp = 0; sp < nsplit; ++sp) L = fmaf(Ls[sp * G + g], fast_exp2(Ms[sp * G + g] - M), L);
        float4 acc = part[i4];
        for (int k = 1; k < SG; ++k) {
            const float4 v = part[k * NQ + i4];
            acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
        if (L > 0.f) r = make_float4(acc.x / L, acc.y / L, acc.z / L, acc.w / L);
        reinterpret_cast<float4*>(O)[i4] = r;
    }
    if (tid == 0) *counter = 0u;  // every sibling has arrived: leave the counter reusable
}

// ------------------------------------------------------------------ work schedule
// The units are the (sequence, KV head) pairs u = b * H_kv + h, laid end to end as one
// array of cache blocks (unit u holds ceil(ctx_b / block_size) of them, starting at
// P[b] + h * nblk_b with P the prefix over sequences of nblk * H_kv). CTA i streams blocks
// [i c, (i+1) c) of that array, c = max(chunk_min, ceil(total / gridDim.x)), so every CTA
// gets the same number of blocks whatever the context lengths. A CTA's range covers pieces
// of one or more units; a unit cut by CTA boundaries is merged by log-sum-exp from its
// pieces, which sit in workspace rows (CTA index + unit index): along the chain of pieces
// that sum grows by at least one per piece, so the rows are distinct and fewer than
// gridDim.x + units.
struct DAItem {
    int b, h;        // sequence, KV head
    int lo, hi;      // cache blocks [lo, hi) of the unit
    int ctx;         // the sequence's context length
    int split, nsplit, slot0;
};

struct DASched {
    int pos, end, c, b;  // flattened block range of this CTA; chunk; current sequence

    // warp 0: clamped context lengths and the block prefix P[0..B] into shared memory
    __device__ __forceinline__ static void scan(const DecodeAttnParams& p, int* P_s, int* ctx_s, int lane,
                                                bool report) {
        constexpr int PER = DA_MAX_B / 32;
        int nb[PER];
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            const int b = k * 32 + lane;
            nb[k] = 0;
            if (b < p.B) {
                const int ctx = da_context(p, b, report);
                ctx_s[b] = ctx;
                const int nblk = (ctx + p.block_size - 1) / p.block_size;
                nb[k] = (nblk > 0 ? nblk + p.unit_cost : 0) * p.H_kv;
            }
        }
        int carry = 0;
        if (lane == 0) P_s[0] = 0;
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            if (k * 32 >= p.B) break;
            int v = nb[k];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += t;
            }
            if (k * 32 + lane < p.B) P_s[k * 32 + lane + 1] = carry + v;
            carry += __shfl_sync(0xffffffffu, v, 31);
        }
    }

    __device__ __forceinline__ void init(const DecodeAttnParams& p, const int* P_s) {
        if (p.unit_mode) {  // P_s[1] holds this unit's block count
            b = (int)blockIdx.x / p.H_kv;
            pos = 0;
            end = P_s[1];
            c = 0;
            return;
        }
        const int total = P_s[p.B];
        c = max(p.chunk_min, (total + (int)gridDim.x - 1) / (int)gridDim.x);
        pos = min(total, (int)blockIdx.x * c);
        end = min(total, pos + c);
        // first sequence whose blocks reach past pos
        int lo = 0, hi = p.B;  // P_s[lo] <= pos < P_s[hi] when pos < total
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (P_s[mid] <= pos) lo = mid; else hi = mid;
        }
        b = lo;
    }

    __device__ __forceinline__ bool next(const DecodeAttnParams& p, const int* P_s, const int* ctx_s, DAItem& it) {
        if (pos >= end) return false;
        if (c == 0) {  // unit mode: the whole unit, one piece
            it.b = b;
            it.h = (int)blockIdx.x % p.H_kv;
            it.lo = 0;
            it.hi = end;
            it.ctx = ctx_s[0];
            it.split = 0;
            it.nsplit = 1;
            it.slot0 = 0;
            pos = end;
            return true;
        }
        // Each unit occupies unit_cost cost-only positions before its blocks, so a CTA that
        // starts (and merges) a unit streams correspondingly fewer blocks; a range holding
        // only such positions of a unit has no piece of it.
        while (pos < end) {
            while (P_s[b + 1] <= pos) ++b;  // skips empty sequences
            const int nbv = (P_s[b + 1] - P_s[b]) / p.H_kv;  // positions per unit of sequence b
            const int rel = pos - P_s[b];
            const int h = rel / nbv;
            const int vlo = rel - h * nbv;
            const int vhi = min(nbv, vlo + (end - pos));
            pos += vhi - vlo;
            const int lo = max(0, vlo - p.unit_cost), hi = max(0, vhi - p.unit_cost);
            if (hi <= lo) continue;
            const int nb = nbv - p.unit_cost;
            it.b = b;
            it.h = h;
            it.lo = lo;
            it.hi = hi;
            it.ctx = ctx_s[b];
            const int off = P_s[b] + h * nbv + p.unit_cost;  // the unit's first block in the array
            const int first = off / c;
            it.nsplit = (off + nb - 1) / c - first + 1;
            it.split = (int)blockIdx.x - first;
            it.slot0 = first + b * p.H_kv + h;
            return true;
        }
        return false;
    }
};

// ------------------------------------------------------------------ the kernel
// Grid: the balanced schedule's CTAs (or one per unit in unit mode). Warp 8 produces the
// tiles of the CTA's items in order into the ring; warps 0..7 consume them, and at the end
// of each item merge their partial softmax states through the ring stage of the item's last
// tile, which they release only after the merge, so the producer keeps streaming the next
// item into the other stages meanwhile.
// TMA = true: the producer's lane 0 moves each cache block of a tile with two 3-D TMA loads
// (box head_dim x 1 head x block_size tokens of a tensor map over [P * block_size, H_kv,
// head_dim]) into the same dense rows, completion counted in bytes on the stage's barrier;
// used when tiles hold whole blocks and the pool size is known. Otherwise the warp gathers
// rows with cp.async.
template <int G, int D, typename KV, bool TMA>
__global__ void __launch_bounds__(DA_NT, (da_minb<G, D, KV>()))
decode_attn_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                   const DecodeAttnParams p) {
    using C = DACfg<G, D, KV>;
    extern __shared__ __align__(1024) unsigned char smem[];
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    int* P_s = reinterpret_cast<int*>(smem + C::OFF_P);
    int* ctx_s = reinterpret_cast<int*>(smem + C::OFF_CTX);
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
    griddep_wait();  // everything above touches only this CTA's shared memory
    griddep_launch();
    if (p.unit_mode) {
        if (tid == 0) {
            const int b = (int)blockIdx.x / p.H_kv;
            const int ctx = da_context(p, b, (int)blockIdx.x % p.H_kv == 0);
            ctx_s[0] = ctx;
            P_s[0] = 0;
            P_s[1] = (ctx + p.block_size - 1) / p.block_size;
        }
    } else if (warp == 0) {
        DASched::scan(p, P_s, ctx_s, lane, blockIdx.x == 0);
    }
    __syncthreads();

    DASched sc;
    sc.init(p, P_s);
    // empty contexts: O = 0 (reference reduce writes o * 0, 13_decode_attn.cuh:48-52)
    if (p.unit_mode) {
        if (sc.end == 0) {
            float* O = p.O + ((size_t)sc.b * p.H_q + ((int)blockIdx.x % p.H_kv) * G) * D;
            for (int i = tid; i < G * D; i += DA_NT) O[i] = 0.f;
        }
    } else {
        for (int b = blockIdx.x; b < p.B; b += gridDim.x)
            if (ctx_s[b] == 0) {
                float* O = p.O + (size_t)b * p.H_q * D;
                for (int i = tid; i < p.H_q * D; i += DA_NT) O[i] = 0.f;
            }
    }
    if (sc.pos >= sc.end) return;  // no blocks for this CTA

    const int bs = p.block_size;
    if (warp == DA_NW) {
        // ------------------------------------------------------------ producer warp
        // Each item's slice of the block table is staged in shared memory, so no tile waits on
        // a dependent global load (slices longer than BT_CAP blocks are read from global).
        int* bt_s = reinterpret_cast<int*>(smem + C::OFF_BT);
        const uint64_t pol = policy_evict_first();
        if (TMA && lane == 0) {
            prefetch_tensormap(&kmap);
            prefetch_tensormap(&vmap);
        }
        int issued = 0;  // tiles whose copies were all requested
        bool ok = true;
        DAItem it;
        while (ok && sc.next(p, P_s, ctx_s, it)) {
            const int* btg = p.block_table + (size_t)it.b * p.num_blocks_per_seq;
            const int nbt = it.hi - it.lo;
            const bool staged = nbt <= C::BT_CAP;
            __syncwarp();  // the previous item's slice is no longer read
            if (staged) {
                for (int j = lane; j < nbt; j += 32) bt_s[j] = btg[it.lo + j];
                __syncwarp();
            }
            const int tok_begin = it.lo * bs;
            const int tok_end = min(it.ctx, it.hi * bs);
            const int ntiles = (tok_end - tok_begin + C::T - 1) / C::T;
            if constexpr (TMA) {
                if (lane == 0) {
                    const uint32_t block_bytes = (uint32_t)(bs * C::ROW);
                    for (int i = 0; i < ntiles; ++i) {
                        const int st = issued % C::STAGES;
                        if (issued >= C::STAGES &&
                            (misc[0] != 0 || !mbar_wait(empty_bar(st), ((issued / C::STAGES) - 1) & 1, p.err))) {
                            misc[0] = 1;
                            ok = false;
                            break;
                        }
                        const int t0 = tok_begin + i * C::T;
                        const int n = min(C::T, tok_end - t0);
                        const int nb = (n + bs - 1) / bs;  // whole blocks (the last may run past the context)
                        const uint32_t sK = ring + st * C::STAGE;
                        mbar_arrive_expect_tx(full_bar(st), 2u * nb * block_bytes);
                        for (int j = 0; j < nb; ++j) {
                            const int blk = t0 / bs + j;
                            int phys = staged ? bt_s[blk - it.lo] : btg[blk];
                            if ((unsigned)phys >= (unsigned)p.num_phys_blocks) {
                                raise_error(p.err, B2_DEVERR_BLOCK_RANGE);
                                phys = 0;
                            }
                            tma_load_3d(sK + j * block_bytes, &kmap, 0, it.h, phys * bs, full_bar(st), pol);
                            tma_load_3d(sK + C::T * C::ROW + j * block_bytes, &vmap, 0, it.h, phys * bs,
                                        full_bar(st), pol);
                        }
                        ++issued;
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            } else {
                for (int i = 0; i < ntiles; ++i) {
                    const int st = issued % C::STAGES;
                    if (issued >= C::STAGES) {
                        const uint32_t par = ((issued / C::STAGES) - 1) & 1;
                        bool w_ok = misc[0] == 0 && mbar_wait(empty_bar(st), par, p.err);
                        w_ok = __shfl_sync(0xffffffffu, w_ok ? 1 : 0, 0) != 0;
                        if (!w_ok) {
                            if (lane == 0) misc[0] = 1;
                            ok = false;
                            break;
                        }
                    }
                    const uint32_t sK = ring + st * C::STAGE;
                    da_issue_tile<C>(p, it.b, it.h, tok_begin, tok_end, i, sK, sK + C::T * C::ROW, bt_s, staged,
                                     lane, pol);
                    cp_async_mbar_arrive_noinc(full_bar(st));
                    ++issued;
                }
            }
        }
        if constexpr (TMA) {
            // drain: the last fill of every stage this thread requested has landed before
            // the CTA can exit, also when a consumer gave up waiting on one
            if (lane == 0)
                for (int j = max(0, issued - C::STAGES); j < issued; ++j)
                    mbar_wait_drain(full_bar(j % C::STAGES), (j / C::STAGES) & 1);
        } else {
            cp_async_wait_all();  // nothing may still be landing in the ring when the warp exits
        }
        return;
    }

    // ---------------------------------------------------------------- consumer warps
    constexpr int NC = DA_NW * 32;
    float* xw = reinterpret_cast<float*>(smem + C::OFF_X) + warp * DA_XW;  // [0,NV) p, [32,32+G) alpha
    float* ml_s = reinterpret_cast<float*>(smem + C::OFF_ML);           // [NW][G][2]
    DAWarp<G, D, KV> w;
    int used = 0;  // tiles consumed
    DAItem it;
    while (sc.next(p, P_s, ctx_s, it)) {
        w.begin(p, it.b, it.h * G, lane);
        const int tok_begin = it.lo * bs;
        const int tok_end = min(it.ctx, it.hi * bs);
        const int ntiles = (tok_end - tok_begin + C::T - 1) / C::T;
        int st = 0;
        for (int i = 0; i < ntiles; ++i, ++used) {
            st = used % C::STAGES;
            const int n = min(C::T, tok_end - (tok_begin + i * C::T));
            if (misc[0] == 0) {
                if (!mbar_wait(full_bar(st), (used / C::STAGES) & 1, p.err)) misc[0] = 1;
            }
            const unsigned char* Kt = smem + st * C::STAGE;
            w.tile(Kt, Kt + C::T * C::ROW, n, warp, lane, xw);
            __syncwarp();
            if (i + 1 < ntiles && lane == 0) mbar_arrive(empty_bar(st));
        }

        // ---- merge the 8 warps through the stage of the item's last tile (still held)
        const float l_tot = w.l_total();
        named_barrier(1, NC);  // every warp is done reading the stage
        float* red = reinterpret_cast<float*>(smem + st * C::STAGE);  // [NW][G][D]
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
        // a wait that gave up sets the error bit and leaves O untouched; the decision is
        // taken on the barrier's OR so that every consumer thread takes the same branch
        const bool abort = named_barrier_or(1, NC, misc[0] != 0);
        if (!abort) {
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
                    const float sc2 = fast_exp2(mw - M);
                    o = fmaf(red[v * G * D + i], sc2, o);
                    L = fmaf(ml_s[(v * G + g) * 2 + 1], sc2, L);
                }
            };
            da_finish<G, D, NC>(p, it.b, it.h, it.split, it.nsplit, it.slot0, tid, misc + 1, red, merge_warps);
        }
        // The stage is refilled only after all 8 warps released it, and ml_s is next written
        // after the next item's first barrier, which every warp reaches only when done here.
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(st));
        if (abort) break;
    }
}

// Two units per CTA (unit mode, TMA producer only): consumer warps 0-3 serve unit
// 2 * blockIdx.x and warps 4-7 unit 2 * blockIdx.x + 1, each group through its own half of
// the ring with its own barriers; lanes 0 and 1 of the producer warp feed the two groups
// independently. For short units (a few hundred tokens) whose count exceeds one wave of
// CTAs: the GPU streams every unit at once instead of in 1.7 waves.
template <int G, int D, typename KV>
__global__ void __launch_bounds__(DA_NT, (da_minb<G, D, KV>()))
decode_attn_pair_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                        const DecodeAttnParams p) {
    using C = DACfg<G, D, KV, 2>;
    constexpr int NWG = C::NWG;
    constexpr int NCG = NWG * 32;
    extern __shared__ __align__(1024) unsigned char smem[];
    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    int* ctx_s = reinterpret_cast<int*>(smem + C::OFF_CTX);  // [2] context of each group's unit (-1: none)
    volatile unsigned int* misc = reinterpret_cast<volatile unsigned int*>(smem + C::OFF_MISC);
    const uint32_t bar0 = smem_u32(smem + C::OFF_BAR);
    auto full_bar = [&](int gr, int s) { return bar0 + 8u * (gr * C::STAGES + s); };
    auto empty_bar = [&](int gr, int s) { return bar0 + 8u * (2 * C::STAGES + gr * C::STAGES + s); };
    auto stage = [&](int gr, int s) { return (gr * C::STAGES + s) * C::STAGE; };
    const int U = p.B * p.H_kv;

    if (tid == 0) {
        for (int gr = 0; gr < 2; ++gr)
            for (int s = 0; s < C::STAGES; ++s) {
                mbar_init(full_bar(gr, s), 1);
                mbar_init(empty_bar(gr, s), NWG);
            }
        misc[0] = 0;  // abort flag
        misc[1] = 0;  // merge tickets (one per group; unused: a unit is never cut here)
        misc[2] = 0;
        fence_mbar_init();
    }
    if (!p.kv_early) {
        griddep_wait();  // everything above touches only this CTA's shared memory
        griddep_launch();
    }
    if (tid < 2) {
        const int u = (int)blockIdx.x * 2 + tid;
        ctx_s[tid] = u < U ? da_context(p, u / p.H_kv, u % p.H_kv == 0) : -1;
    }
    __syncthreads();
    if (p.kv_early && warp != DA_NW) {  // consumers read Q and write O: after the previous grid
        griddep_wait();
        griddep_launch();
    }
    // empty contexts: O = 0 (reference reduce writes o * 0, 13_decode_attn.cuh:48-52)
    for (int gr = 0; gr < 2; ++gr)
        if (ctx_s[gr] == 0) {
            const int u = (int)blockIdx.x * 2 + gr;
            float* O = p.O + ((size_t)(u / p.H_kv) * p.H_q + (u % p.H_kv) * G) * D;
            for (int i = tid; i < G * D; i += DA_NT) O[i] = 0.f;
        }

    const int bs = p.block_size;
    if (warp == DA_NW) {
        // ------------------------------------------------------------ producer lanes 0, 1
        if (lane < 2 && ctx_s[lane] > 0) {
            const int gr = lane;
            const int u = (int)blockIdx.x * 2 + gr;
            const int b = u / p.H_kv, h = u % p.H_kv;
            const int ctx = ctx_s[gr];
            const int nb = (ctx + bs - 1) / bs;
            const int* btg = p.block_table + (size_t)b * p.num_blocks_per_seq;
            int* bt_s = reinterpret_cast<int*>(smem + C::OFF_BT) + gr * (C::BT_CAP / 2);
            const bool staged = nb <= C::BT_CAP / 2;
            if (staged)
                for (int j = 0; j < nb; ++j) bt_s[j] = btg[j];  // independent loads, one latency
            prefetch_tensormap(&kmap);
            prefetch_tensormap(&vmap);
            const uint64_t pol = policy_evict_first();
            const uint32_t block_bytes = (uint32_t)(bs * C::ROW);
            const uint32_t ring = smem_u32(smem);
            const int ntiles = (ctx + C::T - 1) / C::T;
            int issued = 0;
            bool waited = !p.kv_early;
            for (int i = 0; i < ntiles; ++i) {
                const int st = i % C::STAGES;
                if (i >= C::STAGES &&
                    (misc[0] != 0 || !mbar_wait(empty_bar(gr, st), ((i / C::STAGES) - 1) & 1, p.err))) {
                    misc[0] = 1;
                    break;
                }
                const int t0 = i * C::T;
                if (!waited && t0 + C::T >= ctx) {  // this tile holds the newest token's block
                    griddep_wait();
                    waited = true;
                }
                const int n = min(C::T, ctx - t0);
                const int nbt = (n + bs - 1) / bs;
                const uint32_t sK = ring + stage(gr, st);
                mbar_arrive_expect_tx(full_bar(gr, st), 2u * nbt * block_bytes);
                for (int j = 0; j < nbt; ++j) {
                    const int blk = t0 / bs + j;
                    int phys = staged ? bt_s[blk] : btg[blk];
                    if ((unsigned)phys >= (unsigned)p.num_phys_blocks) {
                        raise_error(p.err, B2_DEVERR_BLOCK_RANGE);
                        phys = 0;
                    }
                    tma_load_3d(sK + j * block_bytes, &kmap, 0, h, phys * bs, full_bar(gr, st), pol);
                    tma_load_3d(sK + C::T * C::ROW + j * block_bytes, &vmap, 0, h, phys * bs, full_bar(gr, st), pol);
                }
                issued = i + 1;
            }
            // drain: the last fill of every stage requested has landed before exit
            for (int j = max(0, issued - C::STAGES); j < issued; ++j)
                mbar_wait_drain(full_bar(gr, j % C::STAGES), (j / C::STAGES) & 1);
        }
        return;
    }

    // ---------------------------------------------------------------- consumer groups
    const int gr = warp / NWG;
    const int wl = warp - gr * NWG;
    const int ctx = ctx_s[gr];
    if (ctx <= 0) return;  // the whole group leaves together
    const int u = (int)blockIdx.x * 2 + gr;
    const int b = u / p.H_kv, h = u % p.H_kv;
    float* xw = reinterpret_cast<float*>(smem + C::OFF_X) + warp * DA_XW;  // [0,NV) p, [32,32+G) alpha
    float* ml_s = reinterpret_cast<float*>(smem + C::OFF_ML);           // [NW][G][2]
    DAWarp<G, D, KV, 2> w;
    w.begin(p, b, h * G, lane);
    const int ntiles = (ctx + C::T - 1) / C::T;
    int st = 0;
    for (int i = 0; i < ntiles; ++i) {
        st = i % C::STAGES;
        const int n = min(C::T, ctx - i * C::T);
        if (misc[0] == 0) {
            if (!mbar_wait(full_bar(gr, st), (i / C::STAGES) & 1, p.err)) misc[0] = 1;
        }
        const unsigned char* Kt = smem + stage(gr, st);
        w.tile(Kt, Kt + C::T * C::ROW, n, wl, lane, xw);
        __syncwarp();
        if (i + 1 < ntiles && lane == 0) mbar_arrive(empty_bar(gr, st));
    }
    // merge the group's warps through the stage of its last tile (still held)
    const float l_tot = w.l_total();
    named_barrier(1 + gr, NCG);
    float* red = reinterpret_cast<float*>(smem + stage(gr, st));  // [NWG][G][D]
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < DAWarp<G, D, KV, 2>::VP; ++j) {
            red[(wl * G + g) * D + lane * C::VPL + 2 * j] = w.acc[g][j].x;
            red[(wl * G + g) * D + lane * C::VPL + 2 * j + 1] = w.acc[g][j].y;
        }
    if (w.owner && w.my_t == 0) {
        ml_s[(warp * G + w.my_g) * 2] = w.m_run;
        ml_s[(warp * G + w.my_g) * 2 + 1] = l_tot;
    }
    const bool abort = named_barrier_or(1 + gr, NCG, misc[0] != 0);
    if (!abort) {
        auto merge_warps = [&](int i, float& o, float& M, float& L) {
            const int g = i / D;
            M = -INFINITY;
#pragma unroll
            for (int v = 0; v < NWG; ++v) M = fmaxf(M, ml_s[((gr * NWG + v) * G + g) * 2]);
            o = 0.f;
            L = 0.f;
            if (M == -INFINITY) return;
#pragma unroll
            for (int v = 0; v < NWG; ++v) {
                const float mw = ml_s[((gr * NWG + v) * G + g) * 2];
                if (mw == -INFINITY) continue;
                const float sc2 = fast_exp2(mw - M);
                o = fmaf(red[v * G * D + i], sc2, o);
                L = fmaf(ml_s[((gr * NWG + v) * G + g) * 2 + 1], sc2, L);
            }
        };
        da_finish<G, D, NCG>(p, b, h, 0, 1, 0, tid - gr * NCG, misc + 1 + gr, red, merge_warps);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar(gr, st));
}

// ------------------------------------------------------------------ host side

// Schedule of one launch (at most DA_MAX_B sequences). Balanced: `grid` CTAs, each streaming
// an equal share of the batch's cache blocks (at least chunk_min of them), found on the device
// from the actual context lengths; a unit cut across CTAs is merged through the workspace.
// Unit mode: one CTA per (sequence, KV head), no workspace; used when the workspace cannot
// hold the balanced plan's pieces.
struct AttnPlan {
    int grid;
    int unit_mode;
    int chunk_min;
    int unit_cost;  // cost-only blocks charged per unit (balanced schedule)
    int pair;  // unit mode with two units per CTA (decode_attn_pair_kernel), when TMA is usable
};

// CTAs resident per SM (the kernel's launch bounds, da_minb; D = 0: the largest count, which
// sizes the workspace for every variant)
static int da_ctas_per_sm(int G, int D = 0) {
    if (G >= 8) return 2;
    return (G == 4 && D == 128) ? 2 : DA_MINB;
}

// Bytes of one workspace piece (da_piece_floats) and of the counters of U units.
static size_t da_piece_bytes(int G, int D) { return (size_t)(G * D + ((2 * G + 3) & ~3)) * sizeof(float); }
static size_t da_counter_bytes(long long U) { return ((size_t)U * sizeof(unsigned int) + 255) & ~(size_t)255; }

// A CTA streams at least 128 tokens (and 2 blocks): below that its start-up and merge cost
// more than the parallelism gains (config 1, B1 H12 ctx 1024: 64-token CTAs 7.2 us,
// 128-token 7.1 us, 256-token 8.9 us).
static int da_chunk_min(int block_size) { return std::max(2, (128 + block_size - 1) / block_size); }

// Balanced grid wanted for a launch of Bc sequences: one CTA per resident slot, fewer when
// the longest possible batch has fewer chunks.
static long long da_grid_wanted(int Bc, int H_kv, int G, int max_ctx, int block_size, int num_sms, int D = 0) {
    const long long max_blocks = std::max(1, (max_ctx + block_size - 1) / block_size);
    const long long chunks = ((long long)Bc * H_kv * max_blocks + da_chunk_min(block_size) - 1) / da_chunk_min(block_size);
    // the final merge stages (M, L) of up to gridDim.x pieces per head in one 32 KB ring stage
    const long long merge_cap = 3584 / G;  // 2 grid G floats of (M, L) + 4 KB of partial sums
    // one wave: 1.5, 2 and 3 waves of smaller CTAs measured 4-18% slower (config 3 and its
    // 4- and 8-way head shards), each CTA adding its start-up and merge
    const long long slots = (long long)da_ctas_per_sm(G, D) * num_sms;
    return std::max(1LL, std::min<long long>(std::min<long long>(slots, chunks), merge_cap));
}

static AttnPlan plan_attn(int Bc, int H_kv, int G, int D, int kv_bytes, int max_ctx, int block_size,
                          size_t ws_bytes, int num_sms) {
    static const bool force_unit = getenv("B2_ATTN_PLAN") && strcmp(getenv("B2_ATTN_PLAN"), "unit") == 0;
    const long long U = (long long)Bc * H_kv;
    const long long want = da_grid_wanted(Bc, H_kv, G, max_ctx, block_size, num_sms, D);
    const size_t cnt = da_counter_bytes(U);
    const long long cap = ws_bytes > cnt ? (long long)((ws_bytes - cnt) / da_piece_bytes(G, D)) : 0;
    AttnPlan pl;
    pl.chunk_min = da_chunk_min(block_size);
    // A CTA spends ~4 us starting and merging each unit it touches (q load, warp merge,
    // partial write, fence and ticket), about what it streams of ~56 KB of K+V at its
    // one-CTA-per-slot share of HBM: that many blocks are charged per unit (8-way head shard
    // of config 3: 36.3 -> 34.8 us; CTAs holding two units no longer finish last). Taking
    // the tickets in one batch at the end of each CTA instead was measured slower (36.1 us,
    // config 3 bf16 146 -> 151 us): the final merges then all land in the kernel's tail.
    const int block_bytes = 2 * block_size * D * kv_bytes;
    // Charged only when the grid fills every slot: a narrower grid (short batches such as
    // config 1) gives each CTA more than a slot's share, and there the charge cut pieces
    // finer than the units' own shape (config 1: 10.7 us with it, 8.9 without).
    pl.unit_cost = want >= (long long)da_ctas_per_sm(G, D) * num_sms
                       ? std::max(0, (56 * 1024 + block_bytes / 2) / block_bytes) : 0;
    // Short units that fill the GPU 1.5 times or more by themselves run one CTA per unit:
    // cutting and grouping them costs more in item merges than the last wave loses (GPT-2
    // Small layer, B64 x 12 heads, contexts 129-256 with max_context_len 1024: 16.1-21.4 us
    // per launch one CTA per unit, 19.1-25.0 us balanced).
    const long long max_blocks = std::max(1, (max_ctx + block_size - 1) / block_size);
    const bool short_units = max_blocks <= 64 && 2 * U >= 3LL * da_ctas_per_sm(G, D) * num_sms;
    // balanced when the workspace holds its pieces (grid + U rows) for a grid at least as
    // wide as one CTA per unit would be (or as wanted, when that is narrower)
    const long long g = std::min(want, cap - U);
    pl.pair = 0;
    if (!force_unit && !short_units && g >= std::min(want, U) && g >= 1) {
        pl.grid = (int)g;
        pl.unit_mode = 0;
    } else {
        pl.grid = (int)U;
        pl.unit_mode = 1;
        // short units of head_dim 64 stream two per CTA (one wave instead of 1.5 or more)
        static const bool pair_off = getenv("B2_ATTN_PAIR") && strcmp(getenv("B2_ATTN_PAIR"), "0") == 0;
        pl.pair = short_units && D == 64 && !pair_off;
    }
    return pl;
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
static cudaError_t launch_decode_attn_t(const DecodeAttnParams& prm, const AttnPlan& pl, cudaStream_t st) {
    using C = DACfg<G, D, KV>;
    CUtensorMap km, vm;
    static const bool tma_off = getenv("B2_ATTN_TMA") && strcmp(getenv("B2_ATTN_TMA"), "0") == 0;
    const bool tma = !tma_off && prm.num_phys_blocks > 0 && prm.block_size <= 256 && C::T % prm.block_size == 0 &&
                     kv_map<KV>(&km, prm.k_cache, (long long)prm.num_phys_blocks * prm.block_size, prm.H_kv, D,
                                prm.block_size) &&
                     kv_map<KV>(&vm, prm.v_cache, (long long)prm.num_phys_blocks * prm.block_size, prm.H_kv, D,
                                prm.block_size);
    if constexpr (D == 64) {  // the pair variant's half tiles need head_dim 64
        using C2 = DACfg<G, D, KV, 2>;
        if (tma && pl.pair && pl.unit_mode && C2::T % prm.block_size == 0) {
            if (!set_smem_attr_once((const void*)decode_attn_pair_kernel<G, D, KV>, C2::SMEM, 0))
                return cudaErrorInvalidValue;
            return launch_kernel(decode_attn_pair_kernel<G, D, KV>, dim3((pl.grid + 1) / 2), dim3(DA_NT),
                                 (size_t)C2::SMEM, st, km, vm, prm);
        }
    }
    if (tma) {
        if (!set_smem_attr_once((const void*)decode_attn_kernel<G, D, KV, true>, C::SMEM, 0)) return cudaErrorInvalidValue;
        return launch_kernel(decode_attn_kernel<G, D, KV, true>, dim3(pl.grid), dim3(DA_NT), (size_t)C::SMEM, st, km,
                             vm, prm);
    }
    memset(&km, 0, sizeof(km));
    if (!set_smem_attr_once((const void*)decode_attn_kernel<G, D, KV, false>, C::SMEM, 0)) return cudaErrorInvalidValue;
    return launch_kernel(decode_attn_kernel<G, D, KV, false>, dim3(pl.grid), dim3(DA_NT), (size_t)C::SMEM, st, km, km,
                         prm);
}

template <int D, typename KV>
static cudaError_t dispatch_group(int G, const DecodeAttnParams& prm, const AttnPlan& pl, cudaStream_t st) {
    switch (G) {
        case 1: return launch_decode_attn_t<1, D, KV>(prm, pl, st);
        case 2: return launch_decode_attn_t<2, D, KV>(prm, pl, st);
        case 4: return launch_decode_attn_t<4, D, KV>(prm, pl, st);
        case 8: return launch_decode_attn_t<8, D, KV>(prm, pl, st);
        default: return cudaErrorInvalidValue;
    }
}

// Workspace layout: the arrival counters of one launch's units (256-byte aligned), then the
// piece rows [grid + units][G][D + 2] f32. Launches of a chunked batch reuse it in stream order.
size_t decode_attn_workspace_size(int B, int H_q, int H_kv, int D, int max_ctx, int block_size) {
    if (B <= 0 || H_kv <= 0 || H_q % H_kv != 0 || block_size <= 0) return 0;
    const int G = H_q / H_kv;
    const int Bc = std::min(B, DA_MAX_B);
    const long long U = (long long)Bc * H_kv;
    const long long g = da_grid_wanted(Bc, H_kv, G, max_ctx, block_size, num_sms_current_device());
    return da_counter_bytes(U) + (size_t)(g + U) * da_piece_bytes(G, D);
}

// Validates, plans and launches (in chunks of DA_MAX_B sequences). `counters_zeroed` false
// makes the launcher clear the counter region first (stream-ordered memset).
// kv_early (decode engine only): see DecodeAttnParams::kv_early.
int decode_attn_launch_ex(const b2_decode_attn_args* a, bool counters_zeroed, bool kv_early, cudaStream_t st) {
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
    if (a->workspace && ((uintptr_t)a->workspace & 255)) return B2_ERR_INVALID;
    const int kvb = a->kv_dtype == B2_KV_F32 ? 4 : 2;
    const int D = a->head_dim;
    const size_t ws_bytes = a->workspace ? a->workspace_bytes : 0;
    const int sms = num_sms_current_device();

    DecodeAttnParams prm;
    prm.k_cache = static_cast<const unsigned char*>(a->k_cache);
    prm.v_cache = static_cast<const unsigned char*>(a->v_cache);
    prm.H_q = a->H_q;
    prm.H_kv = a->H_kv;
    prm.block_size = a->block_size;
    prm.num_blocks_per_seq = a->num_blocks_per_seq;
    prm.num_phys_blocks = a->num_phys_blocks;
    const float scale = a->scale != 0.f ? a->scale : 1.0f / sqrtf((float)D);
    prm.scale_log2 = scale * 1.4426950408889634f;
    prm.err = device_error_ptr();
    bool zeroed = counters_zeroed;
    for (int b0 = 0; b0 < a->B; b0 += DA_MAX_B) {
        const int Bc = std::min(DA_MAX_B, a->B - b0);
        const AttnPlan pl = plan_attn(Bc, a->H_kv, G, D, kvb, a->max_context_len, a->block_size, ws_bytes, sms);
        prm.Q = a->Q + (size_t)b0 * a->H_q * D;
        prm.O = a->O + (size_t)b0 * a->H_q * D;
        prm.block_table = a->block_table + (size_t)b0 * a->num_blocks_per_seq;
        prm.context_lens = a->context_lens + b0;
        prm.B = Bc;
        prm.chunk_min = pl.chunk_min;
        prm.unit_cost = pl.unit_mode ? 0 : pl.unit_cost;
        prm.kv_early = kv_early && pl.unit_mode && pl.pair ? 1 : 0;
        prm.unit_mode = pl.unit_mode;
        prm.ws_partial = nullptr;
        prm.ws_counter = nullptr;
        if (!pl.unit_mode) {
            const size_t cnt = da_counter_bytes((long long)Bc * a->H_kv);
            prm.ws_counter = static_cast<unsigned int*>(a->workspace);
            prm.ws_partial = reinterpret_cast<float*>(static_cast<char*>(a->workspace) + cnt);
            if (!zeroed) {
                // counters end every launch at zero, so one clear serves all chunks
                if (cudaMemsetAsync(a->workspace, 0, cnt, st) != cudaSuccess) return B2_ERR_CUDA;
                zeroed = true;
            }
        }
        cudaError_t e;
        if (D == 64)
            e = kvb == 4 ? dispatch_group<64, float>(G, prm, pl, st)
                         : dispatch_group<64, __nv_bfloat16>(G, prm, pl, st);
        else
            e = kvb == 4 ? dispatch_group<128, float>(G, prm, pl, st)
                         : dispatch_group<128, __nv_bfloat16>(G, prm, pl, st);
        if (e != cudaSuccess) return B2_ERR_CUDA;
    }
    return B2_OK;
}

int decode_attn_launch(const b2_decode_attn_args* a, bool counters_zeroed, cudaStream_t st) {
    return decode_attn_launch_ex(a, counters_zeroed, false, st);
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
    // The schedule is planned against what the fixed array holds: when the balanced plan's
    // pieces do not fit, each (sequence, KV head) runs whole in one CTA, which needs no
    // scratch, so no shape is refused for its size. The arrival counters are cleared with a
    // stream-ordered memset on every call, since the array keeps whatever the previous
    // call left in it.
    return b2::decode_attn_launch(&a, false, static_cast<cudaStream_t>(stream));
}
