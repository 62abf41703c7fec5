// e2e_driver.cpp - greedy decode through the reference's own runtime.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile links this driver twice against
// the reference's unmodified runtime sources (runtime/model.cpp,
// executor.cpp, kv_cache.cpp) and kernels:
//   e2e_ref   with the reference's kernels/attention_decode.cu (engine A);
//   e2e_ours  with this repository's include/attention.cuh first on the
//             include path and libforgert_b200.so in place of
//             attention_decode.cu (engine B: the drop-in).
// It mirrors the decode loop of runtime/main.cpp:196-228 (prefill, then one
// Executor::decode per generated token, Executor::greedy_sample for the
// argmax), minus the tokenizer stub that main.cpp has (main.cpp:74, 100-109).
//
// usage: e2e_xxx <model_dir> <max_seq_len> <n_new> <prompt ids...>
//        [--force <file of token ids>]     teacher-forced: feed these tokens
//        [--dump <file>]                   write every step's fp32 logits
// prints one line per generated token: "<step> <argmax> <top1 - top2 logit>"
#include "executor.h"
#include "kv_cache.h"
#include "model.h"
#include "types.h"

#include <cuda_runtime.h>
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <string>
#include <vector>

static float top2_margin(const fp32* logits_gpu, int vocab, std::FILE* dump) {
    std::vector<float> h(vocab);
    CUDA_CHECK(cudaMemcpy(h.data(), logits_gpu, vocab * sizeof(float), cudaMemcpyDeviceToHost));
    if (dump) std::fwrite(h.data(), sizeof(float), h.size(), dump);
    float a = -1e30f, b = -1e30f;
    for (float x : h) {
        if (x > a) { b = a; a = x; } else if (x > b) { b = x; }
    }
    return a - b;
}

int main(int argc, char** argv) {
    if (argc < 5) {
        std::fprintf(stderr, "usage: %s model_dir max_seq_len n_new ids... [--force file]\n", argv[0]);
        return 2;
    }
    const std::string dir = argv[1];
    const int max_seq = std::atoi(argv[2]);
    const int n_new = std::atoi(argv[3]);
    std::vector<int32_t> prompt;
    std::vector<int32_t> forced;
    std::FILE* dump = nullptr;
    for (int i = 4; i < argc; ++i) {
        if (std::string(argv[i]) == "--dump" && i + 1 < argc) {
            dump = std::fopen(argv[++i], "wb");
        } else if (std::string(argv[i]) == "--force" && i + 1 < argc) {
            std::ifstream f(argv[++i]);
            int32_t t;
            while (f >> t) forced.push_back(t);
        } else {
            prompt.push_back(std::atoi(argv[i]));
        }
    }

    // Qwen2-0.5B architecture.
    ModelConfig cfg;
    cfg.vocab_size = 151936;
    cfg.hidden_size = 896;
    cfg.num_heads = 14;
    cfg.num_kv_heads = 2;
    cfg.num_layers = 24;
    cfg.intermediate_size = 4864;
    cfg.max_seq_len = max_seq;
    cfg.rms_norm_eps = 1e-6f;
    cfg.rope_base = 1000000.0f;
    cfg.rope_scale = 1.0f;
    cfg.tie_embeddings = true;

    auto weights = ModelWeights::load(dir, cfg);
    KVCache kv(weights->cfg);
    Executor ex(weights.get(), &kv);

    fp32* logits = ex.prefill(prompt.data(), (int)prompt.size());
    std::vector<int32_t> toks;
    std::vector<float> margins;
    double decode_s = 0.0;
    for (int step = 0; step < n_new; ++step) {
        margins.push_back(top2_margin(logits, cfg.vocab_size, dump));
        const int32_t tok = ex.greedy_sample(logits);
        toks.push_back(tok);
        if (step + 1 == n_new) break;
        const int32_t next = (step < (int)forced.size()) ? forced[step] : tok;
        CUDA_CHECK(cudaDeviceSynchronize());
        const auto t0 = std::chrono::steady_clock::now();
        logits = ex.decode(next);
        CUDA_CHECK(cudaDeviceSynchronize());
        decode_s += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    }
    for (int i = 0; i < (int)toks.size(); ++i) std::printf("%d %d %.6f\n", i, toks[i], margins[i]);
    // forward time of the decode steps only (the logit copy for the margins
    // and the argmax readback are outside it)
    std::printf("# decode_forward_tok_per_s %.2f\n", (n_new - 1) / std::max(decode_s, 1e-9));
    if (dump) std::fclose(dump);
    return 0;
}
