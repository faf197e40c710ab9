// rubidium/model.h — drop-in for the reference's src/model.h (RubidiumTransformer,
// src/model.h:112-139) over librbk's C ABI.  Header-only C++17; link -lrbk.
//
// A caller written against the reference (src/main.cpp:46-209,
// src/fine_tune.cu:130-293) keeps its calls:
//     RubidiumTransformer model;  model.init(cfg, max_batch);
//     float loss = model.forward(d_tok, d_tgt, B, T);
//     model.backward(d_tok, d_tgt, B, T, 1.0f / (BS * GA));
//     model.clip_gradients(1.0f);
//     model.optimizer_step(step, lr, b1, b2, eps, wd);
// Differences a caller sees: errors throw rubidium::Error (the reference's CE/CB
// macros exit(1)); clip_gradients takes effect inside the next optimizer_step
// (it is fused into the tail); update_loss_scale only reads back the state the
// tail already updated on the device; backward accumulates gradients (the
// optimizer step zeroes them) instead of zeroing them on entry.
#pragma once

#include <cuda_runtime.h>

#include <cstdio>
#include <stdexcept>
#include <string>

#include "../rbk.h"

namespace rubidium {

struct Error : std::runtime_error {
    int status;
    Error(int s, const std::string& what) : std::runtime_error(what + ": " + rbk_last_error()), status(s) {}
};

inline void check(int s, const char* what) {
    if (s != RBK_OK) throw Error(s, what);
}

// ModelConfig (src/model.h:16-24).
struct ModelConfig {
    int V = 32000, T = 512, D = 2048, H = 32, L = 10, FF = 8192, hd = 64;
    bool use_fp16 = true;
    bool use_activation_checkpointing = true;
    int grad_accum_steps = 16;
    void init(int v = 32000, int t = 512, int d = 2048, int h = 32, int l = 10, int ff = 8192) {
        V = v; T = t; D = d; H = h; L = l; FF = ff; hd = d / h;
    }
};

struct LoRAConfig {   // src/lora.h:13-20
    int rank = 16;
    float alpha = 32.0f;
    float scaling() const { return alpha / rank; }
};

struct RubidiumTransformer {
    ModelConfig cfg;
    rbk_model* handle = nullptr;
    cudaStream_t stream = nullptr;     // the reference runs on the legacy default stream
    float loss_scale = 65536.0f;       // mirrors the device scaler (src/model.h:120)
    bool overflow = false;             // last step skipped (src/model.h:121)
    int applied_steps = 0;             // optimizer updates applied (device scaler)
    float pending_clip = 0.0f;

    // init (src/model.cu:17-24): allocate, seed (N(0, 0.02) / LN 1 / biases 0), FP16 copy.
    void init(const ModelConfig& c, int max_batch, uint64_t seed = 42) {
        cfg = c;
        rbk_config lay{c.V, c.T, c.D, c.H, c.L, c.FF};
        rbk_model_opts o{max_batch, c.T, c.use_activation_checkpointing ? 1 : 0, 65536.0f, 2000, 0};
        cudaGetDevice(&o.device);
        check(rbk_model_create(&handle, &lay, &o), "rbk_model_create");
        check(rbk_model_init_weights(handle, seed, 0.02f, stream), "rbk_model_init_weights");
    }
    void allocate_activations(int /*max_BT*/) {}   // sized by init(max_batch)
    void convert_weights_fp32_to_fp16() { check(rbk_model_sync_fp16(handle, stream), "rbk_model_sync_fp16"); }

    // forward (src/model.h:130): returns the mean loss (synchronises, as the reference does).
    float forward(const int* d_tokens, const int* d_targets, int B, int T) {
        void* p = nullptr;
        int64_t n = 0;
        check(rbk_model_buffer(handle, RBK_BUF_LOSS, &p, &n), "rbk_model_buffer");
        check(rbk_model_forward(handle, d_tokens, d_targets, B, T, static_cast<float*>(p), stream),
              "rbk_model_forward");
        float loss = 0.0f;
        if (d_targets) {
            if (cudaMemcpyAsync(&loss, p, sizeof(float), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
                cudaStreamSynchronize(stream) != cudaSuccess)
                throw Error(RBK_ERR_CUDA, "loss read-back");
        }
        return loss;
    }
    // backward (src/model.h:131): `loss_scale_arg` is the reference's upstream factor.
    void backward(const int* d_tokens, const int* d_targets, int B, int T, float loss_scale_arg) {
        check(rbk_model_backward(handle, d_tokens, d_targets, B, T, loss_scale_arg, stream), "rbk_model_backward");
    }
    // clip_gradients (src/model.h:133): per-tensor L2 clip, applied inside the next optimizer_step.
    void clip_gradients(float max_norm) { pending_clip = max_norm; }
    // optimizer_step (src/model.h:132): overflow check + unscale + clip + AdamW + FP16 copy + skip.
    void optimizer_step(int t, float lr, float b1, float b2, float eps, float wd) {
        check(rbk_model_optimizer_step(handle, t, lr, b1, b2, eps, wd, pending_clip, stream),
              "rbk_model_optimizer_step");
        pending_clip = 0.0f;
    }
    // update_loss_scale (src/model.h:134): the tail already updated the scaler; read it back.
    void update_loss_scale(bool /*overflow*/) {
        rbk_scaler* dev = nullptr;
        check(rbk_model_scaler(handle, &dev), "rbk_model_scaler");
        rbk_scaler s{};
        if (cudaMemcpyAsync(&s, dev, sizeof(s), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
            cudaStreamSynchronize(stream) != cudaSuccess)
            throw Error(RBK_ERR_CUDA, "scaler read-back");
        loss_scale = s.scale;
        overflow = s.skipped != 0;
        applied_steps = s.applied_steps;
    }
    // save / load (src/model.h:136-137): the reference's RBN2 file plus masters, Adam moments and
    // the loss scaler (rbk_model_save / rbk_model_load).  char_map is the file's 256-entry
    // character-to-token map (the reference stores its tokenizer's char_to_id there).  load on a
    // model that was never init()ed takes the config from the file and sizes the activations for
    // max_batch_on_load sequences of cfg.T tokens.
    int char_map[256] = {};
    int max_batch_on_load = 1;
    void save(const char* path) {
        check(rbk_model_save(handle, path, char_map, stream), "rbk_model_save");
    }
    void load(const char* path) {
        if (!handle) {
            int hdr[7] = {};                 // magic + V T D H L FF
            FILE* f = std::fopen(path, "rb");
            const bool ok = f && std::fread(hdr, sizeof(int), 7, f) == 7;
            if (f) std::fclose(f);
            if (!ok) throw Error(RBK_ERR_IO, std::string("cannot read the header of ") + path);
            ModelConfig c;
            c.init(hdr[1], hdr[2], hdr[3], hdr[4], hdr[5], hdr[6]);
            init(c, max_batch_on_load);
        }
        check(rbk_model_load(handle, path, char_map, stream), "rbk_model_load");
        update_loss_scale(false);
    }
    // The whole trainer loop of src/main.cpp:125-175 on the device (rbk_model_train): the token
    // stream stays resident (d_stream, n tokens), windows are drawn on the device from `seed`,
    // nothing synchronises until the per-step losses are read back at the end.
    void train(const int* d_stream, int64_t n, int steps, int GA, int BS, int max_steps, int warmup, float lr,
               float b1, float b2, float eps, float wd, float gc, float* losses, uint64_t seed = 1) {
        rbk_train_args a{};
        a.tokens = d_stream; a.n_tokens = n; a.starts = nullptr; a.seed = seed;
        a.steps = steps; a.ga = GA; a.B = BS; a.T = cfg.T; a.first_step = applied_steps + 1;
        a.max_steps = max_steps; a.warmup = warmup;
        a.lr = lr; a.b1 = b1; a.b2 = b2; a.eps = eps; a.wd = wd; a.clip = gc;
        a.grad_scale = 1.0f / (BS * GA);      // the reference's backward factor (src/main.cpp:158)
        a.losses = losses;
        check(rbk_model_train(handle, &a, stream), "rbk_model_train");
        update_loss_scale(false);
    }
    // LoRA hooks (src/lora.h:223-231).
    void init_lora(const LoRAConfig& lc, uint64_t seed = 7) {
        check(rbk_model_lora_enable(handle, lc.rank, lc.alpha, seed, stream), "rbk_model_lora_enable");
    }
    void lora_optimizer_step(int t, float lr, float b1, float b2, float eps, float wd) {
        check(rbk_model_lora_step(handle, t, lr, b1, b2, eps, wd, stream), "rbk_model_lora_step");
    }
    void free_all() {
        if (handle) rbk_model_destroy(handle);
        handle = nullptr;
    }
    ~RubidiumTransformer() { free_all(); }
};

}  // namespace rubidium
