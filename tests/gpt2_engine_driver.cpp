// A caller of the reference's GPT2Engine API (the call pattern of the reference's
// src/main.cpp bench mode), compiled against include/gpt2_engine.cuh and linked with
// libb2decode.so by tests/test_gpt2_engine_api*.py.
//   gpt2_engine_driver MODEL_DIR MAX_NEW greedy|topk TOKEN... [-- MAX_NEW2 TOKEN...]
// Prints the tokens passed to the callback, one line per generate() call ("tokens: ..."),
// then the metrics of the last call. The part after "--" continues the session
// (reset_kv = false), the reference's continuation mode.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "gpt2_engine.cuh"

int main(int argc, char** argv) {
    if (argc < 5) {
        fprintf(stderr, "usage: %s MODEL_DIR MAX_NEW greedy|topk TOKEN... [-- MAX_NEW2 TOKEN...]\n", argv[0]);
        return 2;
    }
    const std::string model_dir = argv[1];
    const int max_new = atoi(argv[2]);
    const bool greedy = strcmp(argv[3], "greedy") == 0;
    std::vector<int> prompt, prompt2;
    int max_new2 = 0;
    int i = 4;
    for (; i < argc && strcmp(argv[i], "--") != 0; ++i) prompt.push_back(atoi(argv[i]));
    if (i < argc) {
        max_new2 = atoi(argv[i + 1]);
        for (i += 2; i < argc; ++i) prompt2.push_back(atoi(argv[i]));
    }
    try {
        GPT2Engine engine(model_dir);
        printf("config: %d layers, d %d, vocab %d\n", engine.config().n_layers, engine.config().d_model,
               engine.config().vocab_size);
        InferenceMetrics m;
        std::vector<int> out;
        auto cb = [&](int id) { out.push_back(id); };
        engine.generate(prompt, max_new, 0.8f, 40, greedy, cb, m);
        printf("tokens:");
        for (int t : out) printf(" %d", t);
        printf("\nsession %d\n", engine.session_tokens());
        if (!prompt2.empty()) {
            out.clear();
            engine.generate(prompt2, max_new2, 0.8f, 40, greedy, cb, m, /*reset_kv=*/false);
            printf("tokens:");
            for (int t : out) printf(" %d", t);
            printf("\nsession %d\n", engine.session_tokens());
        }
        printf("metrics: generated %d ttft %.3f tpot %.3f tps %.1f p95 %.3f e2e %.3f kv %.2f mbu %.4f\n",
               m.tokens_generated, m.ttft_ms, m.tpot_ms, m.tps, m.itl_p95_ms, m.end_to_end_ms, m.kv_cache_pct,
               m.mbu);
    } catch (const std::exception& e) {
        printf("error: %s\n", e.what());
        return 1;
    }
    return 0;
}
