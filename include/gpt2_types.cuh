// gpt2_types.cuh — the reference's public engine types, for the GPT2Engine drop-in
// (include/gpt2_engine.cuh). Same names, members and member order as the reference's
// include/gpt2_types.cuh:6-90, so its callers (src/main.cpp) compile unchanged; the
// weight-record types describe the on-disk / on-device INT8 format this library consumes.
// The reference's GPT2Weights (a fixed 12-layer array of device pointers) is internal to its
// engine and is not part of this interface.
#pragma once
#include <cstdint>

// Model dimensions (config.json of a model directory).
struct GPT2Config {
    int n_layers;
    int n_heads;
    int d_model;
    int d_ff;
    int vocab_size;
    int max_seq_len;
    int d_head;
};

// One INT8 linear: packed [N, K/4] int32 (byte j of word i = element 4i + j) and an fp32
// per-output-row scale (absmax / 127).
struct QuantWeight {
    int32_t* packed;
    float* scale;
    int N;
    int K;
};

// The device record of one transformer layer.
struct LayerWeights {
    float* ln1_gamma;
    float* ln1_beta;
    QuantWeight qkv;
    float* qkv_bias;
    QuantWeight out;
    float* out_bias;
    float* ln2_gamma;
    float* ln2_beta;
    QuantWeight ffn_up;
    float* ffn_up_bias;
    QuantWeight ffn_down;
    float* ffn_down_bias;
};

// Which implementation runs the linears. This library implements CUSTOM_INT8; CUBLAS_FP32
// (the reference's fp32 comparison backend) is refused at construction.
enum class InferenceBackend { CUSTOM_INT8, CUBLAS_FP32 };

// What GPT2Engine::generate reports (all times in milliseconds).
struct InferenceMetrics {
    float ttft_ms;        // prompt in -> first token chosen
    float tpot_ms;        // mean time per generated token
    float itl_min_ms;     // inter-token latency: min, max, 95th percentile
    float itl_max_ms;
    float itl_p95_ms;
    float tps;            // generated tokens per second
    int tokens_generated;
    int max_tokens;
    float kv_cache_pct;   // share of the sequence's KV blocks in use
    float vram_used_mb;
    float vram_total_mb;
    float mbu;            // memory-bandwidth utilisation of the decode steps
    float end_to_end_ms;
    bool generating;
};
