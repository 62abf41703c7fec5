// e2e_driver.cpp - greedy decode through the reference's own runtime.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile links this driver against the
// reference's unmodified runtime sources (runtime/model.cpp, executor.cpp,
// kv_cache.cpp) and kernels:
//   e2e_ref    with the reference's kernels/attention_decode.cu (engine A);
//   e2e_ours   with this repository's include/attention.cuh first on the
//              include path and libforgert_b200.so in place of
//              attention_decode.cu (engine B: the drop-in);
//   e2e_v3     with the reference's own decode_attn_v3_vec where executor.cpp
//              calls decode_attn_v4_flash (oracle/control_v3/attention.cuh):
//              a control that changes only the attention kernel's rounding;
//   e2e_graph  engine B built with --default-stream per-thread and
//              FORGERT_E2E_GRAPH: the decode step without the per-token host
//              work (see --graph below).
// It mirrors the decode loop of runtime/main.cpp:196-228 (prefill, then one
// Executor::decode per generated token, Executor::greedy_sample for the
// argmax), minus the tokenizer stub that main.cpp has (main.cpp:74, 100-109).
//
// usage: e2e_xxx <model_dir> <max_seq_len> <n_new> <prompt ids...>
//        [--force <file of token ids>]     teacher-forced: feed these tokens
//        [--dump <file>]                   write every step's fp32 logits
//        [--graph]                         (e2e_graph only) one CUDA graph per
//                                          decode position, captured up front:
//                                          token id in by fr_copy_async from
//                                          pinned memory, the 24 layers, the
//                                          reference's argmax, the argmax out
//                                          by fr_copy_async (replacing the
//                                          per-token cudaMalloc, H2D copy and
//                                          synchronous readback of
//                                          runtime/executor.cpp:288-311)
// prints one line per generated token: "<step> <argmax> <top1 - top2 logit>"
// (margin 0 in --graph mode), then the decode rates.
#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <memory>
#include <string>
#include <vector>

#include "kv_cache.h"
#include "model.h"
#include "types.h"
#ifdef FORGERT_E2E_GRAPH
// The graphed step calls Executor::run_forward and sets the stream of its
// cuBLAS handle, both private members of the reference's class: they are
// opened for this test driver only.
#define private public
#endif
#include "executor.h"
#ifdef FORGERT_E2E_GRAPH
#undef private
#include "forgert_attn.h"

// kernels/sampling.cu: the reference's two-phase argmax (executor.cpp:30-31
// declares it the same way)
struct MaxPair { float val; int32_t idx; };
extern void greedy_sample(const float*, MaxPair*, int32_t*, int, cudaStream_t);
#endif

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
    bool graph = false;
    for (int i = 4; i < argc; ++i) {
        if (std::string(argv[i]) == "--graph") {
            graph = true;
        } else if (std::string(argv[i]) == "--dump" && i + 1 < argc) {
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
    double forward_s = 0.0, step_s = 0.0;
    if (graph) {
#ifdef FORGERT_E2E_GRAPH
        // Decode step = one graph per position (the reference bakes kv_pos into
        // its launches), all captured before the timed loop.
        cudaStream_t s = cudaStreamPerThread;
        CUBLAS_CHECK(cublasSetStream(ex.cublas_, s));
        int32_t *tok_in = nullptr, *tok_out = nullptr, *tok_dev = nullptr;
        CUDA_CHECK(cudaHostAlloc(&tok_in, sizeof(int32_t), cudaHostAllocDefault));
        CUDA_CHECK(cudaHostAlloc(&tok_out, sizeof(int32_t), cudaHostAllocDefault));
        CUDA_CHECK(cudaMalloc(&tok_dev, sizeof(int32_t)));
        const int p0 = (int)prompt.size();
        // the split-KV workspace cannot grow inside a capture: size it first
        if (fr_reserve_workspace(fr_decode_workspace_size(1, cfg.num_heads, cfg.num_kv_heads,
                                                          cfg.head_dim(), p0 + n_new)) != FR_OK)
            std::abort();
        std::vector<cudaGraphExec_t> execs(std::max(0, n_new - 1));
        for (int step = 0; step + 1 < n_new; ++step) {
            cudaGraph_t g;
            CUDA_CHECK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
            if (fr_copy_async(tok_dev, tok_in, sizeof(int32_t), s) != FR_OK) std::abort();
            fp32* lg = ex.run_forward(tok_dev, 1, p0 + step, false);
            ::greedy_sample(lg, reinterpret_cast<MaxPair*>(ex.argmax_buf_.ptr),
                            ex.argmax_idx_buf_.as<int32_t>(), cfg.vocab_size, s);
            if (fr_copy_async(tok_out, ex.argmax_idx_buf_.ptr, sizeof(int32_t), s) != FR_OK)
                std::abort();
            CUDA_CHECK(cudaStreamEndCapture(s, &g));
            CUDA_CHECK(cudaGraphInstantiate(&execs[step], g, 0));
            CUDA_CHECK(cudaGraphDestroy(g));
        }
        margins.push_back(0.f);
        int32_t tok = ex.greedy_sample(logits);
        toks.push_back(tok);
        CUDA_CHECK(cudaDeviceSynchronize());
        const auto t0 = std::chrono::steady_clock::now();
        for (int step = 0; step + 1 < n_new; ++step) {
            *tok_in = (step < (int)forced.size()) ? forced[step] : tok;
            CUDA_CHECK(cudaGraphLaunch(execs[step], s));
            CUDA_CHECK(cudaStreamSynchronize(s));
            tok = *tok_out;
            toks.push_back(tok);
            margins.push_back(0.f);
        }
        step_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        forward_s = step_s;
        for (auto& e : execs) cudaGraphExecDestroy(e);
        cudaFreeHost(tok_in);
        cudaFreeHost(tok_out);
        cudaFree(tok_dev);
#else
        std::fprintf(stderr, "--graph needs the e2e_graph build\n");
        return 2;
#endif
    } else {
        for (int step = 0; step < n_new; ++step) {
            // the logit copy for the margins (and the dump) is outside the timed step
            margins.push_back(top2_margin(logits, cfg.vocab_size, dump));
            CUDA_CHECK(cudaDeviceSynchronize());
            const auto t0 = std::chrono::steady_clock::now();
            const int32_t tok = ex.greedy_sample(logits);
            toks.push_back(tok);
            if (step + 1 == n_new) break;
            const int32_t next = (step < (int)forced.size()) ? forced[step] : tok;
            const auto t1 = std::chrono::steady_clock::now();
            logits = ex.decode(next);
            CUDA_CHECK(cudaDeviceSynchronize());
            const auto t2 = std::chrono::steady_clock::now();
            forward_s += std::chrono::duration<double>(t2 - t1).count();
            step_s += std::chrono::duration<double>(t2 - t0).count();
        }
    }
    for (int i = 0; i < (int)toks.size(); ++i) std::printf("%d %d %.6f\n", i, toks[i], margins[i]);
    // forward: Executor::decode (token upload + layers); step: the argmax of
    // the previous logits and its readback + the forward (the reference
    // loop's per-token work; one graph replay in --graph mode)
    std::printf("# decode_forward_tok_per_s %.2f\n", (n_new - 1) / std::max(forward_s, 1e-9));
    std::printf("# decode_step_tok_per_s %.2f\n", (n_new - 1) / std::max(step_s, 1e-9));
    if (dump) std::fclose(dump);
    return 0;
}
