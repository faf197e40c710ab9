// train_main.cpp — the reference trainer loop's shape (src/main.cpp:125-175:
// LR warm-up + cosine, gradient accumulation, clip, optimizer step) driving
// librbk through the C++ drop-in header.  Synthetic tokens; prints one line
// per step.  Build: make -C rubidium-train_b200 examples
//   usage: train_main [steps] [ga] [V T D H L FF B]
//   RBK_LOAD=<file> resumes from a checkpoint (weights, masters, Adam moments,
//   loss scaler; the step count continues); RBK_SAVE=<file> writes one at the end.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

#include "rubidium/model.h"

int main(int argc, char** argv) {
    const int steps = argc > 1 ? atoi(argv[1]) : 4;
    const int GA = argc > 2 ? atoi(argv[2]) : 2;
    rubidium::ModelConfig cfg;
    cfg.init(argc > 3 ? atoi(argv[3]) : 4096, argc > 4 ? atoi(argv[4]) : 128, argc > 5 ? atoi(argv[5]) : 256,
             argc > 6 ? atoi(argv[6]) : 4, argc > 7 ? atoi(argv[7]) : 4, argc > 8 ? atoi(argv[8]) : 1024);
    const int BS = argc > 9 ? atoi(argv[9]) : 8;
    const float lr = 3e-4f, b1 = 0.9f, b2 = 0.999f, eps = 1e-8f, wd = 0.1f, gc = 1.0f;
    const int warmup = 2;
    try {
        rubidium::RubidiumTransformer model;
        model.init(cfg, BS);
        int start = 0;
        if (const char* lp = getenv("RBK_LOAD")) {
            model.load(lp);
            start = model.applied_steps;
            printf("loaded %s: %d steps applied, scale %.0f\n", lp, start, model.loss_scale);
        }
        std::mt19937 gen(42);
        std::uniform_int_distribution<int> tokd(0, cfg.V - 1);
        std::vector<int> h_tok(BS * cfg.T), h_tgt(BS * cfg.T);
        int *d_tok = nullptr, *d_tgt = nullptr;
        cudaMalloc(&d_tok, sizeof(int) * BS * cfg.T);
        cudaMalloc(&d_tgt, sizeof(int) * BS * cfg.T);
        for (int step = start + 1; step <= start + steps; ++step) {
            float lr_t = step < warmup ? lr * step / warmup
                                       : lr * 0.5f * (1.0f + cosf(3.14159265f * (step - warmup) /
                                                                    (start + steps - warmup + 1)));
            float loss_acc = 0.0f;
            for (int ga = 0; ga < GA; ++ga) {
                for (int i = 0; i < BS * cfg.T; ++i) { h_tok[i] = tokd(gen); h_tgt[i] = tokd(gen); }
                cudaMemcpy(d_tok, h_tok.data(), sizeof(int) * BS * cfg.T, cudaMemcpyHostToDevice);
                cudaMemcpy(d_tgt, h_tgt.data(), sizeof(int) * BS * cfg.T, cudaMemcpyHostToDevice);
                loss_acc += model.forward(d_tok, d_tgt, BS, cfg.T);
                model.backward(d_tok, d_tgt, BS, cfg.T, 1.0f / GA);
            }
            model.clip_gradients(gc);
            model.optimizer_step(step, lr_t, b1, b2, eps, wd);
            model.update_loss_scale(false);
            printf("step %d loss %.4f lr %.2e scale %.0f skipped %d\n", step, loss_acc / GA, lr_t, model.loss_scale,
                   (int)model.overflow);
        }
        if (const char* sp = getenv("RBK_SAVE")) {
            model.save(sp);
            printf("saved %s\n", sp);
        }
        cudaFree(d_tok);
        cudaFree(d_tgt);
    } catch (const rubidium::Error& e) {
        fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
    return 0;
}
