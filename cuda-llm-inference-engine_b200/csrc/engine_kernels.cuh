// Launchers of the batched decode-step kernels (engine_kernels.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace b2 {
// Fused QKV split of the decode step (int8_gemm.cu gemm_launch_qkv): q [B, d]; K/V caches
// [P, block_size, H, d_head] (fp32, or bf16 when bf16 != 0) written at each sequence's pos.
struct QkvScatterArgs {
    float* q = nullptr;
    void* k = nullptr;
    void* v = nullptr;
    const int* pos = nullptr;
    const int* block_table = nullptr;
    int d = 0, block_size = 0, nbps = 0, bf16 = 0;
};
int launch_prefill_attention(const int2* items, int n_items, int H, int D, int kv_dtype, const float* q,
                             const void* k_cache, const void* v_cache, const int* block_table, int nbps,
                             int block_size, const int* pos, float* O, cudaStream_t st);
int gemm_launch_qkv(int M, int N, int K, const int32_t* A, const int32_t* BT, const float* sA, const float* sB,
                    const float* bias, const QkvScatterArgs& sc, cudaStream_t st, void* ws = nullptr,
                    size_t ws_bytes = 0);

// keys: [2 * B] argmax keys (approximate, then exact), both zeroed for the step
int launch_embed(int B, int d, const int* tokens, const int* pos, const float* wte, const float* wpe, float* x,
                 int* ctx_lens, unsigned long long* keys, cudaStream_t st);
int launch_ln_quant(int rows, int cols, const float* x, const float* gamma, const float* beta, float eps,
                    int32_t* q, float* scale, float* y, cudaStream_t st, void* y_hi = nullptr,
                    void* y_lo = nullptr);
int launch_split_bf16(const float* x, void* hi, void* lo, size_t n, cudaStream_t st);
// logits [M, N] optional; with cand (int2 [M, cand_cap]) and cand_cnt ([M], zero before the
// step) every logit within cand_delta of its row's running maximum is recorded as
// (value bits, local index) for the exact rescoring
int launch_vocab_bf16x3(int M, int N, int K, const void* h_hi, const void* h_lo, const void* w_hi, const void* w_lo,
                        float* logits, unsigned long long* keys, cudaStream_t st, int n_offset = 0,
                        float cand_delta = 0.f, int* cand_cnt = nullptr, void* cand = nullptr, int cand_cap = 0);
int launch_qkv_scatter(int B, int d, int H, int dh, int block_size, int nbps, const float* qkv, const int* pos,
                       const int* block_table, float* q, void* k_cache, void* v_cache, int kv_dtype, cudaStream_t st);
int launch_vocab_argmax(int B, int V, int d, const float* h, const float* wte, float* logits,
                        unsigned long long* keys, cudaStream_t st);
// exact fp32 rescoring of the argmax candidates of the tensor-core vocab projection: keys
// [B] approximate (read), keys_exact [B] (written), the candidate record of
// launch_vocab_bf16x3 (read, counts reset to zero); logits optional
int launch_vocab_rescore(int B, int V, int d, int n_offset, const float* h, const float* wte, float delta,
                         float* logits, const unsigned long long* keys, unsigned long long* keys_exact,
                         int* cand_cnt, const void* cand, int cand_cap, cudaStream_t st);
// max_v ||w_v||_2 over the rows of w [V, d] (synchronous; < 0 on failure)
float row_norm_max(int V, int d, const float* w);
int launch_advance(int B, const unsigned long long* keys, int* tokens, int* pos, const int* forced,
                   const int* forced_len, int forced_stride, int* out_tokens, int out_stride, int max_pos,
                   cudaStream_t st, int* next_out = nullptr);
int launch_rowmax(int rows, int cols, const float* x, float* amax, cudaStream_t st);
int launch_quantize_scaled(int rows, int cols, const float* x, const float* amax, int32_t* q, float* scale,
                           cudaStream_t st);
int launch_dequant_residual(int M, int N, const int32_t* acc, const float* sA, const float* sB, const float* bias,
                            const float* residual, float* out, cudaStream_t st);
}  // namespace b2
