// GPT2Engine (include/gpt2_engine.cuh): the reference's single-sequence generation API over
// the batched decode engine (include/b2engine.h) at batch 1. Host code only.
//
// Reference behaviour followed (src/gpt2_engine.cu:622-783, src/sampler.cu):
//   - fresh session: the whole prompt is processed, then each step feeds the last chosen
//     token; here the prompt goes through b2_engine_prefill (all tokens but the last in one
//     pass) and its last token through one decode step;
//   - continuation (reset_kv = false on a live session): each prompt token is fed through the
//     decode path at the next position;
//   - the loop stops before passing the end-of-text token 50256 to the callback, and after
//     max_new_tokens tokens; metrics as the reference's InferenceMetrics.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <numeric>
#include <stdexcept>
#include <string>

#include "b2engine.h"
#include "gpt2_engine.cuh"

namespace {

constexpr int kEndOfText = 50256;          // GPT-2's <|endoftext|>, where the reference stops
constexpr double kHbmBytesPerS = 7.7e12;   // B200 HBM3e bandwidth, the denominator of mbu

void check(int status, const char* what) {
    if (status != B2_OK) throw std::runtime_error(std::string(what) + ": " + b2_status_string(status));
}

double now_ms() {
    using namespace std::chrono;
    return duration<double, std::milli>(steady_clock::now().time_since_epoch()).count();
}

}  // namespace

GPT2Engine::GPT2Engine(const std::string& model_dir, InferenceBackend backend) : config_{} {
    if (backend != InferenceBackend::CUSTOM_INT8)
        throw std::runtime_error("GPT2Engine: only the INT8 backend is implemented on this library");
    b2_engine* e = nullptr;
    check(b2_engine_load(model_dir.c_str(), /*max_batch=*/1, B2_KV_F32, &e), "b2_engine_load");
    engine_ = e;
    b2_gpt2_config c{};
    b2_engine_config(engine_, &c);
    config_ = GPT2Config{c.n_layers, c.n_heads, c.d_model, c.d_ff, c.vocab_size, c.max_seq_len, c.d_head};
}

GPT2Engine::~GPT2Engine() {
    if (engine_) b2_engine_destroy(engine_);
}

void GPT2Engine::reset_session() { current_pos_ = 0; }

int GPT2Engine::step(int token) {
    int32_t in = token, next = -1;
    check(b2_engine_decode_step(engine_, &in, &next, nullptr), "b2_engine_decode_step");
    ++current_pos_;
    return next;
}

// The k largest logits of the last step, softmax at `temperature`, one uniform draw against
// the cumulative probabilities; the generator (C rand) is reseeded whenever the seed changes,
// as the reference's sampler does.
int GPT2Engine::sample_top_k(int k, float temperature, unsigned int seed) {
    const int V = config_.vocab_size;
    logits_.resize(V);
    check(b2_engine_read_logits(engine_, logits_.data()), "b2_engine_read_logits");
    k = std::max(1, std::min(k, V));
    std::vector<int> idx(V);
    std::iota(idx.begin(), idx.end(), 0);
    std::partial_sort(idx.begin(), idx.begin() + k, idx.end(),
                      [&](int a, int b) { return logits_[a] > logits_[b]; });
    const float top = logits_[idx[0]];
    std::vector<float> p(k);
    float sum = 0.f;
    for (int i = 0; i < k; ++i) {
        p[i] = expf((logits_[idx[i]] - top) / temperature);
        sum += p[i];
    }
    for (float& x : p) x /= sum;
    if (seed != last_seed_) {
        srand(seed);
        last_seed_ = seed;
    }
    const float r = (float)rand() / RAND_MAX;
    float cum = 0.f;
    for (int i = 0; i < k; ++i) {
        cum += p[i];
        if (r < cum) return idx[i];
    }
    return idx[k - 1];
}

void GPT2Engine::generate(const std::vector<int>& prompt_tokens, int max_new_tokens, float temperature, int top_k,
                          bool greedy, std::function<void(int)> token_callback, InferenceMetrics& metrics,
                          bool reset_kv) {
    const int pl = (int)prompt_tokens.size();
    metrics = InferenceMetrics{};
    metrics.max_tokens = max_new_tokens;
    metrics.generating = true;
    if (pl < 1) throw std::invalid_argument("GPT2Engine::generate: empty prompt");
    if (reset_kv) reset_session();
    if (current_pos_ + pl > config_.max_seq_len)
        throw std::invalid_argument("GPT2Engine::generate: prompt beyond max_seq_len");
    if (!greedy && !logits_on_) {
        check(b2_engine_keep_logits(engine_, 1, nullptr), "b2_engine_keep_logits");
        logits_on_ = true;
    }
    const double t0 = now_ms();
    int next;
    if (current_pos_ == 0) {
        check(b2_engine_start(engine_, 1, prompt_tokens.data(), &pl, pl, config_.max_seq_len - pl, 0),
              "b2_engine_start");
        check(b2_engine_prefill(engine_, nullptr), "b2_engine_prefill");
        current_pos_ = pl - 1;
        next = step(prompt_tokens[pl - 1]);
    } else {
        next = -1;
        for (int t : prompt_tokens) next = step(t);
    }
    unsigned int seed = 42u;
    if (!greedy) next = sample_top_k(top_k, temperature, seed);
    metrics.ttft_ms = (float)(now_ms() - t0);

    // bytes a decode step reads at batch 1: int8 weights, their scales and biases, the tied
    // embedding (as two bf16 halves), and the K and V of the live context (fp32)
    const GPT2Config& c = config_;
    const double lin = (double)c.n_layers * (4.0 * c.d_model * c.d_model + 2.0 * c.d_model * c.d_ff);
    const double fixed = lin + 4.0 * c.vocab_size * c.d_model;
    const int max_blocks = (c.max_seq_len + 15) / 16;
    std::vector<float> itl;
    double total_ms = 0.0;
    int generated = 0;
    for (int s = 0; s < max_new_tokens; ++s) {
        if (next == kEndOfText || current_pos_ >= c.max_seq_len) break;
        token_callback(next);
        metrics.tokens_generated = ++generated;
        const double ts = now_ms();
        next = step(next);
        if (!greedy) next = sample_top_k(top_k, temperature, ++seed);
        const double ms = now_ms() - ts;
        itl.push_back((float)ms);
        total_ms += ms;
        metrics.tpot_ms = (float)(total_ms / generated);
        metrics.tps = (float)(1000.0 * generated / total_ms);
        metrics.itl_min_ms = *std::min_element(itl.begin(), itl.end());
        metrics.itl_max_ms = *std::max_element(itl.begin(), itl.end());
        if (itl.size() >= 20) {
            std::vector<float> sorted = itl;
            std::sort(sorted.begin(), sorted.end());
            metrics.itl_p95_ms = sorted[(size_t)(sorted.size() * 0.95)];
        } else {
            metrics.itl_p95_ms = metrics.itl_max_ms;
        }
        metrics.kv_cache_pct = 100.0f * ((current_pos_ + 15) / 16) / max_blocks;
        size_t free_b = 0, total_b = 0;
        if (cudaMemGetInfo(&free_b, &total_b) == cudaSuccess) {
            metrics.vram_used_mb = (float)((total_b - free_b) / (1024.0 * 1024.0));
            metrics.vram_total_mb = (float)(total_b / (1024.0 * 1024.0));
        }
        const double step_bytes = fixed + 8.0 * c.n_layers * (double)current_pos_ * c.d_model;
        metrics.mbu = (float)(metrics.tps * step_bytes / kHbmBytesPerS);
    }
    metrics.end_to_end_ms = (float)(now_ms() - t0);
    metrics.generating = false;
}
