/*
 * b2engine.h — C ABI of the batched GPT-2 INT8 decode engine on B200.
 *
 * Replaces the decode path of the reference's GPT2Engine (src/gpt2_engine.cuh:9-92,
 * src/gpt2_engine.cu:447-528 forward_layer, :716-776 decode loop), which runs one sequence,
 * blocks on host<->device copies several times per layer and samples on the host. Here one
 * decode step advances every sequence of a batch by one token entirely on the device:
 * embedding, per layer [LayerNorm+quantise, INT8 QKV (+bias), QKV split + paged KV write,
 * K13 decode attention, quantise, INT8 out-proj (+bias+residual), LayerNorm+quantise, INT8
 * FC1 (+bias+GELU), quantise, INT8 FC2 (+bias+residual)], final LayerNorm, tied vocab
 * projection (tensor cores, then every argmax candidate recomputed exactly in the reference's
 * fp32 order) with a GPU argmax (lowest index on ties, like the reference's std::max_element,
 * src/sampler.cu:10-14), and the position advance. LayerNorm sums in the reference kernel's
 * order and the INT8 GEMM epilogues are bit-exact, so the int8 activations equal the
 * reference engine's wherever the attention outputs (summed in another order) round alike. A step is a fixed launch sequence, so
 * b2_engine_run_steps replays it as a CUDA graph.
 *
 * Formats kept from the reference: the on-disk model directory (config.json + *.bin,
 * python/export_gpt2.py:59-187, src/gpt2_engine.cu:41-112), QuantWeight packing
 * (include/gpt2_types.cuh:16-21), and the paged KV layout [P, 16, H, d_head] per layer
 * (src/gpt2_engine.cu:143-153) with per-sequence block tables.
 */
#ifndef B2ENGINE_H
#define B2ENGINE_H

#include <stddef.h>
#include <stdint.h>
#include "b2decode.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Same fields and order as the reference's GPT2Config (include/gpt2_types.cuh:6-14). */
typedef struct {
    int n_layers, n_heads, d_model, d_ff, vocab_size, max_seq_len, d_head;
} b2_gpt2_config;

typedef struct b2_engine b2_engine;

/* Engine with seeded random weights: N(0, 0.02) for wte, wpe, every linear weight (then
 * per-row int8 quantised) and every bias; LayerNorm gamma = 1, beta = 0. max_batch
 * sequences of up to cfg->max_seq_len tokens get KV blocks from the engine's pool. */
int b2_engine_create_random(const b2_gpt2_config* cfg, int max_batch, int kv_dtype, uint64_t seed,
                            b2_engine** out);

/* Writes an NCCL unique id (ncclGetUniqueId) for b2_engine_create_random_tp into out[bytes >= 128]. */
int b2_nccl_unique_id(void* out, size_t bytes);

/* Tensor-parallel engine, rank `rank` of `world` (one process per GPU, the GPU current when
 * called): heads, QKV and FC1 output columns and vocab rows are split across ranks; out-proj
 * and FC2 are row-parallel. Every rank draws the full model with the same seeds as
 * b2_engine_create_random and keeps its slice, so the sharded engine computes the same model.
 * The row-parallel inputs are quantised with the global row scale (all-reduce max of the
 * per-rank absmax), the int32 partial products are all-reduced exactly before the
 * dequantisation epilogue, and the greedy argmax is an all-reduce(max) of 64-bit keys, so the
 * int8 bytes and int32 accumulators equal the single-GPU ones. nccl_id comes from rank 0's
 * b2_nccl_unique_id, shared by the caller. Requires n_heads and d_ff divisible by world. */
int b2_engine_create_random_tp(const b2_gpt2_config* cfg, int max_batch, int kv_dtype, uint64_t seed,
                               const void* nccl_id, int rank, int world, b2_engine** out);

/* Engine from a model directory in the reference's format (GPT2Engine::load_weights,
 * src/gpt2_engine.cu:75-112). Any number of layers. Missing or short files are errors. */
int b2_engine_load(const char* model_dir, int max_batch, int kv_dtype, b2_engine** out);

/* Writes the engine's weights in the reference's directory format. */
int b2_engine_export(const b2_engine* e, const char* model_dir);

void b2_engine_destroy(b2_engine* e);

int b2_engine_config(const b2_engine* e, b2_gpt2_config* out);

/* Starts `batch` sequences: prompts_host [batch, prompt_stride] token ids, prompt_lens_host
 * [batch] (>= 1). Frees the previous sequences' KV blocks, gives every sequence
 * ceil(max_seq_len / 16) blocks from the pool's free list (seed 0: in pool order, like the
 * reference engine; any other seed: a seeded random order, so block tables are scattered over
 * the pool), and sets every position to 0. Positions stop at
 * max_seq_len - 1 (further steps rewrite that slot). Steps then
 * feed the prompt token by token through the decode path (the reference's continuation
 * mode, src/gpt2_engine.cu:683-696) and continue greedily. Synchronous. */
int b2_engine_start(b2_engine* e, int batch, const int32_t* prompts_host, const int32_t* prompt_lens_host,
                    int prompt_stride, int max_new_tokens, uint64_t seed);

/* Batched prefill, right after b2_engine_start: every prompt token but each sequence's last
 * runs through the layer stack in one pass (8192 tokens per pass; longer prompts in several),
 * one row per token: LayerNorm+quantise, one QKV GEMM over all rows with the K/V written to
 * each token's cache slot, attention of each row over its own prefix, and the MLP; then every
 * sequence waits at its last prompt token, so the next step predicts the first new token.
 * Same K/V and states as prompt_len - 1 decode steps (attention splits may merge in another
 * order: logits agree to ~1e-6 relative), except that the per-position predictions of those
 * steps are not recorded. Under tensor parallelism every rank calls it. Synchronous. */
int b2_engine_prefill(b2_engine* e, b2_stream_t stream);

/* One decode step for every active sequence (asynchronous on `stream`). */
int b2_engine_step(b2_engine* e, b2_stream_t stream);

/* `steps` decode steps, replayed from a CUDA graph of one step captured on first use. */
int b2_engine_run_steps(b2_engine* e, int steps, b2_stream_t stream);

/* One decode step with tokens chosen by the caller: tokens_in[b] (b < the batch given to
 * b2_engine_start) is fed at sequence b's current position, the step runs (graph replay, as
 * b2_engine_run_steps), every position advances by one, and the greedy next token of each
 * sequence is written to next_out[b] (NULL: not copied). This is the reference's decode
 * loop body (src/gpt2_engine.cu:716-750: copy the token in, embed, layers, final LayerNorm,
 * logits, argmax) for a whole batch, with the token supplied by the caller instead of taken
 * from the engine's own argmax or prompt; use it for teacher forcing, host-side sampling or
 * continuation prompts. tokens_in and next_out may be device or host pointers (copied with
 * cudaMemcpyDefault on `stream`; with pageable host memory the copies are synchronous).
 * Asynchronous otherwise. */
int b2_engine_decode_step(b2_engine* e, const int32_t* tokens_in, int32_t* next_out, b2_stream_t stream);

/* Runs one decode step eagerly on a private stream with a CUDA event before every launch and
 * writes a text breakdown into report[report_bytes]: a first line "step_us <total> launches
 * <n>", then one line per kernel class "<label> <launches> <total µs> <share %>", largest
 * first. The events serialise the launches, so the total is somewhat above a graph replay's.
 * Under tensor parallelism every rank must call it for the same step. Synchronous. */
int b2_engine_profile_step(b2_engine* e, char* report, size_t report_bytes);

/* Copies the greedy token chosen at each position: out_host [batch, out_stride], entry
 * [b][p] = argmax after the step at position p-1 (-1 where no step has run). Synchronous. */
int b2_engine_read_tokens(const b2_engine* e, int32_t* out_host, int out_stride);

/* Keeps the fp32 logits [batch, vocab] of the last step on the device (tests); returns the
 * device pointer through *logits, or NULL when disabled. */
int b2_engine_keep_logits(b2_engine* e, int enable, const float** logits);

/* Copies the last step's logits [batch, vocab] to host memory (needs keep_logits). Synchronous. */
int b2_engine_read_logits(const b2_engine* e, float* out_host);

/* Failure path of the tensor-parallel scale exchange, for diagnostics and tests (no
 * counterpart in the reference, which has no multi-GPU path). Runs the row-parallel
 * quantiser that the out-projection and FC2 use under tensor parallelism (one CTA per row:
 * row maximum published to every rank, then a bounded wait for every rank's) as rank 0 of a
 * 2-rank group whose rank 1 never arrives. xchg_self and xchg_absent are zeroed device
 * regions of b2_tp_exchange_bytes(rows) bytes; the second stands in for the absent rank's.
 * Each row's wait gives up after its bound (2 s), sets B2_DEVERR_TIMEOUT in the device error
 * word and the kernel finishes with this rank's own row maxima, so the context stays usable.
 * x [rows, cols] fp32 (cols % 4 == 0, rows <= 256); q_packed [rows, cols/4]; scales [rows].
 * Asynchronous on `stream`. */
size_t b2_tp_exchange_bytes(int rows);
int b2_tp_quantize_absent_peer(int rows, int cols, const float* x, int32_t* q_packed, float* scales,
                               void* xchg_self, void* xchg_absent, b2_stream_t stream);

/* Synthetic context: fills the whole KV pool with seeded N(0,1) values and moves every
 * sequence to position ctx_len (< max_seq_len), as if ctx_len tokens had been decoded. For
 * benchmarks of long contexts without a prefill. Synchronous. */
int b2_engine_fill_kv_random(b2_engine* e, int ctx_len, uint64_t seed);

/* Current position of every sequence (tokens already in its KV cache). Synchronous. */
int b2_engine_positions(const b2_engine* e, int32_t* pos_host);

#ifdef __cplusplus
}
#endif

#endif /* B2ENGINE_H */
