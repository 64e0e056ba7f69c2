// Exposes the reference's own GPT2Engine (src/gpt2_engine.cu, INT8 backend), compiled
// unchanged from its sources where they lie, to the tests as an oracle (test infrastructure
// only; built by oracle/build_ref.sh into oracle/_ref/libref_engine.so).
//
// ref_engine_generate runs GPT2Engine(model_dir) and generate(prompt, max_new, greedy) and
// returns the generated tokens plus, per token, the logits that chose it. The logits live in
// the engine's private d_logits_ buffer; generate() calls the token callback with each token
// right after the argmax that picked it and before the next step overwrites the buffer, so
// the callback copies the buffer then (the class's member names are made reachable from
// this file by compiling its header with `private` defined as `public`, which changes no
// layout or behaviour). The final token of a run (chosen after the last callback) is read
// the same way after generate() returns. Only the extern "C" ref_* symbols are exported.
#define private public
#include "gpt2_engine.cuh"
#undef private
#include "timer.cuh"

#include <algorithm>
#include <vector>

#define REF_API extern "C" __attribute__((visibility("default")))

// Returns the number of tokens written to out_tokens (<= max_new + 1): the reference stops
// early at its end-of-text token 50256, which is then the last one written.
// out_logits: [max_new + 1, vocab] or NULL.
// token_by_token != 0 feeds the prompt through the reference's decode path instead of its
// FlashAttention prefill: generate(prompt[0]) with no new tokens on a fresh session, then
// generate(prompt[1:], reset_kv = false), the engine's continuation mode
// (src/gpt2_engine.cu:683-696).
REF_API int ref_engine_generate(const char* model_dir, const int* prompt, int prompt_len, int max_new,
                                int* out_tokens, float* out_logits, int token_by_token) {
    GPT2Engine eng(model_dir);
    const int V = eng.config().vocab_size;
    int n = 0;
    InferenceMetrics m{};
    auto grab = [&](int tok) {
        out_tokens[n] = tok;
        if (out_logits)
            cudaMemcpy(out_logits + (size_t)n * V, eng.d_logits_, (size_t)V * sizeof(float), cudaMemcpyDeviceToHost);
        ++n;
    };
    if (token_by_token && prompt_len > 1) {
        std::vector<int> first(prompt, prompt + 1), rest(prompt + 1, prompt + prompt_len);
        eng.generate(first, 0, 1.0f, 1, /*greedy=*/true, [](int) {}, m, /*reset_kv=*/true);
        eng.generate(rest, max_new, 1.0f, 1, /*greedy=*/true, grab, m, /*reset_kv=*/false);
    } else {
        std::vector<int> toks(prompt, prompt + prompt_len);
        eng.generate(toks, max_new, 1.0f, 1, /*greedy=*/true, grab, m, /*reset_kv=*/true);
    }
    // the last token chosen (after the final step, or the end-of-text token that stopped the
    // loop): generate returns before calling back with it
    {
        std::vector<float> h(V);
        cudaMemcpy(h.data(), eng.d_logits_, (size_t)V * sizeof(float), cudaMemcpyDeviceToHost);
        const int tok = (int)(std::max_element(h.begin(), h.end()) - h.begin());
        out_tokens[n] = tok;
        if (out_logits) std::copy(h.begin(), h.end(), out_logits + (size_t)n * V);
        ++n;
    }
    return cudaDeviceSynchronize() == cudaSuccess ? n : -1;
}
