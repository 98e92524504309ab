// Drives the forge:: C++ engines for tests/test_forge_engine.py:
//   forge_engine_driver <model.squeeze> <max_new> [q=Q,K,V,O,GATE,UP,DOWN,EMB] <prompt tokens...>
// (q=: the file's quantization types for forge::BatchEngine, default all Q8)
// prints "engine: <tokens>" from forge::Engine::generate (greedy) and
// "batch <i>: <tokens>" from forge::BatchEngine::generate with the same
// prompt twice plus a shifted copy, then "forward: <argmax>".
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "forge/batch_engine.hpp"
#include "forge/engine.hpp"

int main(int argc, char** argv) {
    if (argc < 4) return 2;
    const uint32_t max_new = (uint32_t)std::atoi(argv[2]);
    int qt[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int first = 3;
    if (argv[3][0] == 'q' && argv[3][1] == '=') {
        const char* s = argv[3] + 2;
        for (int i = 0; i < 8 && *s; i++) {
            qt[i] = std::atoi(s);
            while (*s && *s != ',') s++;
            if (*s == ',') s++;
        }
        first = 4;
    }
    std::vector<int32_t> prompt;
    for (int i = first; i < argc; i++) prompt.push_back(std::atoi(argv[i]));

    forge::Engine e;
    e.set_max_context(512);
    if (!e.load_model(argv[1])) {
        std::printf("load failed: %s\n", e.last_error().c_str());
        return 1;
    }
    forge::GenerationResult r = e.generate(prompt, max_new);
    std::printf("engine:");
    for (size_t i = prompt.size(); i < r.tokens.size(); i++) std::printf(" %d", r.tokens[i]);
    std::printf("\naccepted %d rejected %d tps %.1f mem %zu\n", r.mtp_accepted, r.mtp_rejected, r.tokens_per_second,
                r.peak_memory_bytes);

    std::vector<float> lg = e.forward(prompt);
    std::printf("forward: %d %zu\n", lg.empty() ? -1 : e.sample_greedy(lg.data(), (uint32_t)lg.size()), lg.size());

    forge::BatchConfig bc;
    bc.model = e.config();
    bc.max_context = 512;
    bc.model.kv_cache_size = 512;
    for (int i = 0; i < 7; i++) bc.qtype[i] = qt[i];
    bc.emb_qtype = qt[7];
    forge::BatchEngine b(bc, 3, 512, 0);
    if (!b.ok() || !b.load_squeeze(argv[1])) {
        std::printf("batch load failed: %s\n", b.last_error().c_str());
        return 1;
    }
    std::vector<int32_t> other = prompt;
    for (auto& t : other) t = (t + 7) % (int32_t)bc.model.n_vocab;
    std::vector<std::vector<int32_t>> out;
    if (!b.generate({prompt, other, prompt}, max_new, &out)) {
        std::printf("batch generate failed: %s\n", b.last_error().c_str());
        return 1;
    }
    for (size_t i = 0; i < out.size(); i++) {
        std::printf("batch %zu:", i);
        for (int32_t t : out[i]) std::printf(" %d", t);
        std::printf("\n");
    }
    return 0;
}
