/*
 * b2decode.h — C ABI of the B200 (sm_100a) GPT-2 decode hot path.
 *
 * Two kernels families sit behind this boundary:
 *   - K13: split-K paged decode attention (one query token per sequence) over a
 *     paged KV cache addressed through a per-sequence block table;
 *   - K14: per-row symmetric INT8 quantizer and INT8 x INT8 -> INT32 GEMM with a fused
 *     dequantisation epilogue (plain / +bias / +bias+GELU / +bias+residual).
 *
 * Conventions (all entry points):
 *   - every pointer is a DEVICE pointer owned by the caller; nothing here allocates;
 *   - work is enqueued asynchronously on `stream` (NULL = legacy default stream);
 *   - every entry returns a b2_status; shapes the kernels do not support are errors,
 *     never silent no-ops;
 *   - faults detected on the device (a wait that timed out, a context length beyond its
 *     block-table row, a block-table entry outside the pool) are recorded as bits in a
 *     device error word, read with b2_get_device_error().
 *
 * Layouts are the reference's (mohith-suresh/CUDA-LLM-Inference-Engine):
 *   Q, O            [B, H_q, 1, head_dim] fp32                      (kernels/decode/13_decode_attn.cuh:34)
 *   k/v cache       [num_phys_blocks, block_size, H_kv, head_dim]  (kernels/decode/13_decode_attn.cuh:35-36)
 *   block_table     [B, num_blocks_per_seq] int32                  (kernels/decode/13_decode_attn.cuh:37)
 *   context_lens    [B] int32, read on the device                   (kernels/decode/13_decode_attn.cuh:38)
 *   int8 operands   [rows, K/4] int32, byte j of word i = element 4i+j (little endian)
 *                                                                   (kernels/quantization/14_int8_gemm.cu:43-58)
 *   scales          [rows] fp32, scale = absmax/127 (1 if the row is all zero)
 *                                                                   (kernels/quantization/14_int8_gemm.cu:36-38)
 */
#ifndef B2DECODE_H
#define B2DECODE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* b2_stream_t; /* a cudaStream_t */

/* Host-side status codes. */
enum {
    B2_OK = 0,
    B2_ERR_INVALID = 1,      /* bad argument: null pointer, negative size, misaligned buffer */
    B2_ERR_UNSUPPORTED = 2,  /* shape the kernels do not implement (e.g. GQA group 3) */
    B2_ERR_WORKSPACE = 3,    /* workspace missing or smaller than the size query returned */
    B2_ERR_CUDA = 4,         /* a CUDA runtime call failed (launch error, bad device) */
    B2_ERR_TIMEOUT = 5       /* a tensor-parallel peer did not answer within its bound */
};

/* Device error bits (b2_get_device_error). */
#define B2_DEVERR_TIMEOUT 1u      /* a bounded wait (mbarrier / flag) gave up */
#define B2_DEVERR_CTX_RANGE 2u    /* context_lens[b] > num_blocks_per_seq * block_size */
#define B2_DEVERR_BLOCK_RANGE 4u  /* block_table entry outside [0, num_phys_blocks) */

/* KV-cache element types. */
enum { B2_KV_F32 = 0, B2_KV_BF16 = 1 };

/* INT8 GEMM epilogues; same order as the reference's `enum class I8Epilogue`
 * (kernels/quantization/14_int8_gemm.cuh:36). */
enum { B2_EPI_PLAIN = 0, B2_EPI_BIAS = 1, B2_EPI_BIAS_GELU = 2, B2_EPI_BIAS_RESIDUAL = 3 };

/* ------------------------------------------------------------------ K13 decode attention */

typedef struct {
    int B, H_q, H_kv, head_dim;      /* head_dim in {64, 128}; H_q / H_kv in {1, 2, 4, 8} */
    const float* Q;                  /* [B, H_q, head_dim] */
    const void* k_cache;             /* [P, block_size, H_kv, head_dim], kv_dtype elements */
    const void* v_cache;
    int kv_dtype;                    /* B2_KV_F32 or B2_KV_BF16 */
    const int* block_table;          /* [B, num_blocks_per_seq] */
    const int* context_lens;         /* [B] (device) */
    int max_context_len;             /* host upper bound of context_lens; sizes the workspace */
    int block_size;                  /* tokens per KV block (engine: 16) */
    int num_blocks_per_seq;          /* block-table row stride */
    int num_phys_blocks;             /* P, for device bounds checks; 0 = unchecked */
    float scale;                     /* softmax scale; 0 = 1/sqrt(head_dim) */
    float* O;                        /* [B, H_q, head_dim] */
    void* workspace;                 /* see b2_decode_attn_workspace_size */
    size_t workspace_bytes;
} b2_decode_attn_args;

/* Bytes of workspace b2_decode_attn needs for these shapes (either KV element type). The
 * kernel gives every CTA an equal share of the batch's cache blocks, found on the device
 * from context_lens, so one (sequence, KV head) may be cut across CTAs; the workspace holds
 * one arrival counter per (sequence, KV head) of a launch (at the start, 256-byte aligned)
 * and the cut pieces' partial results. The counters must be zero before the first call
 * (cudaMemset once); every call leaves them zero again. With no workspace (NULL) or one too
 * small for the balanced schedule, each (sequence, KV head) runs whole in one CTA, which
 * needs none (slower when few long sequences cannot fill the GPU). Batches above 256
 * sequences run as several launches that reuse the workspace.
 * Replaces the caller-side sizing `B*H_q*DA_MAX_SPLITS*(d+2)` floats
 * (reference src/gpt2_engine.cu:156, tests/test_decode_attention.cu:91). */
size_t b2_decode_attn_workspace_size(int B, int H_q, int H_kv, int head_dim,
                                     int max_context_len, int block_size);

/* Split-K paged decode attention, one launch per 256 sequences (split merge fused into the
 * kernel).
 * Replaces run_decode_attn (reference kernels/decode/13_decode_attn.cu:84-109). */
int b2_decode_attn(const b2_decode_attn_args* args, b2_stream_t stream);

/* Capacity of the fixed device scratch array used by b2_decode_attn_noalloc: 16 MiB per GPU. */
#define B2_DECODE_NOALLOC_SCRATCH_BYTES (16u << 20)

/* Decode attention that allocates nothing and needs no caller workspace. No counterpart
 * in the reference: it exists for callers that cannot call cudaMalloc — code running while
 * a CUDA graph is being captured by someone else, allocator-restricted plugin hosts, or
 * real-time loops that forbid allocation after start-up — and that also cannot hand over
 * a workspace buffer of their own.
 *   - The caller still passes Q, the caches, the block table, context_lens and O;
 *     args->workspace and args->workspace_bytes are ignored.
 *   - The workspace is a file-scope device array of B2_DECODE_NOALLOC_SCRATCH_BYTES held by
 *     every GPU that loads the library until the process exits, planned like a caller
 *     workspace of that size: when the balanced schedule's pieces do not fit, each
 *     (sequence, KV head) runs whole in one CTA, which needs none, so no shape is refused
 *     for its size (slower on few long sequences, same results within fp32 rounding).
 *   - The first call on each device looks up the array's device address; make that first
 *     call before any stream capture that should contain this entry point. Each kernel
 *     variant (GQA group, head_dim, KV dtype) also sets its shared-memory limit on its own
 *     first call.
 *   - Every call uses the same array: calls that may overlap on the GPU (different streams,
 *     or different host threads on one device) race on it and must be serialised by the
 *     caller. Each call clears the array's arrival counters itself (a stream-ordered memset).
 *   - Calls no cudaMalloc, cudaFree or allocating library routine. */
int b2_decode_attn_noalloc(const b2_decode_attn_args* args, b2_stream_t stream);

/* ------------------------------------------------------------------ K14 INT8 */

/* Per-row symmetric fp32 -> int8 quantisation, packed 4 per int32, plus fp32 scales.
 * Replaces run_quantize_fp32_to_int8 (reference kernels/quantization/14_int8_gemm.cu:172-180).
 * cols must be a multiple of 4. */
int b2_quantize_fp32_to_int8(int rows, int cols, const float* input, int32_t* output_packed,
                             float* scales, b2_stream_t stream);

/* C[M,N] = epilogue( float(sum_k A[m,k] * BT[n,k]) * scale_A[m] * scale_B[n] ).
 * bias [N] is read for every epilogue but PLAIN; residual [M,N] only for BIAS_RESIDUAL.
 * Replaces run_int8_gemm / _bias / _bias_gelu / _bias_residual
 * (reference kernels/quantization/14_int8_gemm.cu:182-232). K must be a multiple of 4. */
int b2_int8_gemm(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed,
                 const float* scale_A, const float* scale_B, const float* bias,
                 const float* residual, float* C, int epilogue, b2_stream_t stream);

/* Bytes of workspace that let b2_int8_gemm_ws split the K dimension across CTAs for shapes
 * whose output tiles cannot fill the GPU (decode: M = batch); 0 when it would not split.
 * No counterpart in the reference (its dp4a kernel has a fixed 64x64 tile grid). */
/* When M <= 128 and the activation holds >= 256 KB (batch 128 at K >= 2048), the workspace
 * holds the exchange rows of the reduce-scatter split instead: 128-column tiles whose K range
 * is split over a thread-block cluster of 2, 4 or 8 CTAs, each CTA finishing one column slice
 * from its partners' exact int32 partials. */
size_t b2_int8_gemm_workspace_size(int M, int N, int K);

/* b2_int8_gemm with a caller workspace for split-K: each CTA contracts a K range into
 * exact int32 partials, and the last CTA of each tile sums them and runs the epilogue, so
 * results are bit-identical to b2_int8_gemm. The workspace must be zeroed once before first
 * use; every call leaves its arrival counters zero again. Calls sharing a workspace must not
 * overlap on the GPU. */
int b2_int8_gemm_ws(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed,
                    const float* scale_A, const float* scale_B, const float* bias,
                    const float* residual, float* C, int epilogue, void* workspace,
                    size_t workspace_bytes, b2_stream_t stream);

/* Raw int32 accumulators C_acc[M,N] = sum_k A[m,k] * BT[n,k] (no dequantisation): the
 * bit-exact view of the contraction inside the reference's int8_gemm_dp4a_kernel
 * (kernels/quantization/14_int8_gemm.cu:96-140), which the reference never exposes. */
int b2_int8_gemm_s32(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed,
                     int32_t* C_acc, b2_stream_t stream);

/* b2_int8_gemm_s32 with a caller workspace (b2_int8_gemm_workspace_size bytes, 256-byte
 * aligned), as b2_int8_gemm_ws; bit-identical to b2_int8_gemm_s32. */
int b2_int8_gemm_s32_ws(int M, int N, int K, const int32_t* A_packed, const int32_t* BT_packed,
                        int32_t* C_acc, void* workspace, size_t workspace_bytes, b2_stream_t stream);

/* ------------------------------------------------------------------ LayerNorm */

/* Row-wise LayerNorm, optionally fused with the per-row int8 quantiser that follows it in
 * every use of the decode step:
 *   out[r, c] = gamma[c] * (x[r, c] - mean_r) * rsqrtf(var_r + eps) + beta[c]
 * with mean_r and var_r = E[x^2] - mean^2 summed in the order of the reference's 256-thread
 * kernel, so the result is bit-identical to run_layernorm
 * (kernels/layernorm/15_layernorm_residual.cu:59-103, 115-125). When q_packed is not NULL the
 * normalised rows are also quantised exactly as b2_quantize_fp32_to_int8 would
 * (q_packed [rows, cols/4], scales [rows]); out may then be NULL. out may equal x (in place,
 * as the reference engine uses it). cols % 4 == 0, cols <= 8192. */
int b2_layernorm(int rows, int cols, const float* x, const float* gamma, const float* beta, float eps, float* out,
                 int32_t* q_packed, float* scales, b2_stream_t stream);

/* ------------------------------------------------------------------ diagnostics */

/* Returns the device error word of the current device (B2_DEVERR_* bits), synchronising
 * the device first; clears it when clear != 0. */
unsigned int b2_get_device_error(int clear);

/* Status of the last call made through the reference-compatible C++ wrappers, which
 * return void (include/b2_reference_api.h). */
int b2_last_status(void);

const char* b2_status_string(int status);

/* Library ABI version (major * 100 + minor). */
int b2_version(void);

#ifdef __cplusplus
}
#endif

#endif /* B2DECODE_H */
