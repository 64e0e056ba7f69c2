// Peer-memory collectives of the tensor-parallel decode step (tp_collectives.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace b2 {

constexpr int TP_MAX_RANKS = 8;
constexpr int TP_MAX_CTAS = 256;

// Byte offsets inside a rank's exchange region.
struct TpLayout {
    int bmax = 0;          // rows the amax slots hold
    size_t amax = 0;       // f32 [TP_MAX_RANKS][bmax]: row maxima, slot per source rank
    size_t flags = 0;      // u32 [3][TP_MAX_RANKS][TP_MAX_CTAS]: epoch flags written by each source rank
    size_t epochs = 0;     // u32 [2][TP_MAX_CTAS]: this rank's last epoch per kernel and CTA
    size_t bytes = 0;
    static TpLayout make(int bmax) {
        TpLayout L;
        L.bmax = bmax;
        L.amax = 0;
        L.flags = (((size_t)TP_MAX_RANKS * bmax * 4) + 255) & ~(size_t)255;
        L.epochs = L.flags + (size_t)3 * TP_MAX_RANKS * TP_MAX_CTAS * 4;
        L.bytes = L.epochs + (size_t)2 * TP_MAX_CTAS * 4;
        return L;
    }
};

// Every rank's buffers as this rank addresses them (its own, or an IPC mapping of a peer's).
struct TpPeers {
    float* x[TP_MAX_RANKS];              // residual stream [B, d]
    const int32_t* acc[TP_MAX_RANKS];    // int32 partial products [B, d]
    unsigned char* xchg[TP_MAX_RANKS];   // exchange region (TpLayout)
    TpLayout L;
    int rank = 0, world = 1;
    unsigned int* err = nullptr;         // device error word
};

// Row-parallel quantisation with the global row scale: q/scale of x [B, kl] (this rank's columns).
int launch_tp_quantize(int B, int kl, const float* x, int32_t* q, float* scale, const TpPeers& P, cudaStream_t st);
// Sum of every rank's int32 partials, dequant + bias + residual, new residual into every rank's x.
int launch_tp_reduce(int B, int d, const float* sA, const float* sB, const float* bias, const TpPeers& P,
                     cudaStream_t st);

}  // namespace b2
