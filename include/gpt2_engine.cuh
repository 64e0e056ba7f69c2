// gpt2_engine.cuh — GPT2Engine, the reference's single-sequence generation API
// (src/gpt2_engine.cuh:9-29 of mohith-suresh/CUDA-LLM-Inference-Engine), served by this
// library's batched B200 decode engine (include/b2engine.h) with a batch of one.
//
// Same class name, constructor, generate / reset_session / session_tokens / config
// signatures, so the reference's callers (src/main.cpp) compile and link against
// libb2decode.so unchanged. Behaviour:
//   - the constructor loads a model directory in the reference's format; a directory that is
//     missing or short, or the CUBLAS_FP32 backend, throws std::runtime_error (the reference
//     exits the process);
//   - generate(prompt, max_new_tokens, ...) on a fresh session runs the prompt through the
//     batched prefill and continues greedily or by top-k sampling; with reset_kv = false and a
//     live session the prompt tokens extend the session through the decode path (the
//     reference's continuation mode). Generation stops at the end-of-text token 50256 (not
//     passed to the callback), after max_new_tokens, or when the session reaches
//     max_seq_len;
//   - greedy picks the reference's fp32 argmax (lowest index on ties); top-k sampling
//     (temperature, k) follows the reference's sampler (src/sampler.cu:16-45): the k largest
//     logits, softmax at the temperature, one rand() draw against the cumulative sum, seeded
//     42 for the first token and 43, 44, ... after;
//   - the token callback runs on the calling thread after each token is chosen.
// Not thread-safe: one GPT2Engine per thread (the reference's is not either).
#pragma once
#include <functional>
#include <string>
#include <vector>

#include "gpt2_types.cuh"

struct b2_engine;

class GPT2Engine {
public:
    GPT2Engine(const std::string& model_dir, InferenceBackend backend = InferenceBackend::CUSTOM_INT8);
    ~GPT2Engine();
    GPT2Engine(const GPT2Engine&) = delete;
    GPT2Engine& operator=(const GPT2Engine&) = delete;

    void generate(const std::vector<int>& prompt_tokens, int max_new_tokens, float temperature, int top_k,
                  bool greedy, std::function<void(int token_id)> token_callback, InferenceMetrics& metrics,
                  bool reset_kv = true);

    // Clear KV cache / session state. Call between independent conversations.
    void reset_session();

    int session_tokens() const { return current_pos_; }

    const GPT2Config& config() const { return config_; }

private:
    GPT2Config config_;
    b2_engine* engine_ = nullptr;
    int current_pos_ = 0;     // tokens in the session's KV cache
    bool logits_on_ = false;  // logits kept on the device (needed by top-k sampling)
    unsigned int last_seed_ = 0;
    std::vector<float> logits_;

    int step(int token);  // one decode step on `token`; returns the greedy next token
    int sample_top_k(int k, float temperature, unsigned int seed);
};
