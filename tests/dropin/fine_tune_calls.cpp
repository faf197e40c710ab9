// fine_tune_calls.cpp — the model / LoRA call sequence of the reference's LoRA trainer
// (src/fine_tune.cu:179-196,224-253,283-292) written against the drop-in headers under the
// reference's own names ("model.h", "lora.h" from include/rubidium/compat).  The tokenizer
// and instruction-corpus parts of that file are left out: they are not part of librbk.
// A base checkpoint is written first (main-trainer style), then the fine-tune sequence loads
// it, adds rank-r adapters, runs `steps` steps of GA micro-steps and frees everything.
//   usage: fine_tune_calls <checkpoint path> [steps]
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <vector>

#include "lora.h"
#include "model.h"

int main(int argc, char** argv) {
    if (argc < 2) {
        fprintf(stderr, "usage: fine_tune_calls <checkpoint path> [steps]\n");
        return 2;
    }
    const char* ckpt = argv[1];
    const int steps = argc > 2 ? atoi(argv[2]) : 2;
    const int V = 512, T = 64, D = 128, H = 2, L = 2, FF = 256, BS = 2, GA = 2;
    init_handles();
    try {
        {   // the main trainer's set-up and save (src/main.cpp:105-110, :181)
            ModelConfig cfg;
            cfg.init(V, T, D, H, L, FF);
            RubidiumTransformer base;
            base.init(cfg);
            base.allocate_activations(BS * cfg.T);
            std::map<unsigned char, int> c2i;
            std::map<int, unsigned char> i2c;
            for (int c = 'a'; c <= 'z'; ++c) {
                c2i[(unsigned char)c] = c - 'a' + 1;
                i2c[c - 'a' + 1] = (unsigned char)c;
            }
            base.char_to_id = c2i;
            base.id_to_char = i2c;
            base.save(ckpt);
            base.free_all();
        }
        std::vector<int> h_tok(BS * T * 4), h_tgt(BS * T * 4);
        for (size_t i = 0; i < h_tok.size(); ++i) {
            h_tok[i] = (int)((i * 2654435761u) % V);
            h_tgt[i] = (int)((i * 40503u + 7) % V);
        }
        int *d_tokens = nullptr, *d_targets = nullptr;
        CE(cudaMalloc(&d_tokens, h_tok.size() * sizeof(int)));
        CE(cudaMalloc(&d_targets, h_tgt.size() * sizeof(int)));
        CE(cudaMemcpy(d_tokens, h_tok.data(), h_tok.size() * sizeof(int), cudaMemcpyHostToDevice));
        CE(cudaMemcpy(d_targets, h_tgt.data(), h_tgt.size() * sizeof(int), cudaMemcpyHostToDevice));

        RubidiumTransformer model;
        ModelConfig model_cfg;
        model_cfg.init(V, T, D, H, L, FF);
        model.init(model_cfg);
        model.allocate_activations(BS * T);
        model.load(ckpt);
        if (model.char_to_id.size() != 27 || model.id_to_char[1] != 'a') {
            fprintf(stderr, "character map did not survive the checkpoint\n");
            return 1;
        }
        LoRAConfig lora_cfg;
        lora_cfg.rank = 16;
        lora_cfg.alpha = 32.0f;
        lora_cfg.dropout = 0.1f;
        init_lora(model_cfg.D, model_cfg.FF, lora_cfg);
        printf("Base model frozen. LoRA params: ~%.3fM\n", g_lora.count_params() / 1e6);
        const int n = (int)h_tok.size() / T;
        for (int step = 1; step <= steps; ++step) {
            const float lr_t = 1e-3f * step / steps;
            float loss_acc = 0.0f;
            for (int ga = 0; ga < GA; ++ga) {
                const int offset = ((step * GA + ga) % (n - BS + 1)) * T;
                const float loss = model.forward(d_tokens + offset, d_targets + offset, BS, T);
                model.backward(d_tokens + offset, d_targets + offset, BS, T, 1.0f / (BS * GA));
                loss_acc += loss;
            }
            model.clip_gradients(1.0f);
            lora_optimizer_step(step, lr_t, 0.9f, 0.999f, 1e-8f, 0.0f);
            CE(cudaDeviceSynchronize());
            printf("step %d loss %.4f\n", step, loss_acc / GA);
            if (!std::isfinite(loss_acc)) return 1;
        }
        CE(cudaFree(d_tokens));
        CE(cudaFree(d_targets));
        model.free_all();
        lora_free();
    } catch (const rubidium::Error& e) {
        fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
    destroy_handles();
    printf("fine-tune call sequence ok\n");
    return 0;
}
