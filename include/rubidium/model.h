// rubidium/model.h — drop-in for the reference's src/model.h (RubidiumTransformer,
// src/model.h:112-139) and src/lora.h (LoRAConfig, the g_lora state and its free
// functions, src/lora.h:13-20,218-231) over librbk's C ABI.  Header-only C++17;
// link -lrbk -lcudart.
//
// A caller written against the reference (src/main.cpp:46-209,
// src/fine_tune.cu:130-293) keeps its calls:
//     RubidiumTransformer model;
//     model.init(cfg);                         // allocation deferred ...
//     model.allocate_activations(BS * cfg.T);  // ... to here (or to first use)
//     model.char_to_id = c2i; model.id_to_char = i2c;
//     float loss = model.forward(d_tok, d_tgt, B, T);
//     model.backward(d_tok, d_tgt, B, T, 1.0f / (BS * GA));
//     model.clip_gradients(1.0f);
//     model.optimizer_step(step, lr, b1, b2, eps, wd);
//     init_lora(D, FF, lora_cfg); lora_optimizer_step(step, lr, b1, b2, eps, wd); lora_free();
// include/rubidium/compat/{model,lora}.h put these names in the global namespace
// under the reference's own header names, so its sources compile unchanged.
//
// Differences a caller sees: errors throw rubidium::Error (the reference's CE/CB
// macros exit(1)); clip_gradients takes effect inside the next optimizer_step
// (it is fused into the tail); update_loss_scale only reads back the state the
// tail already updated on the device; backward accumulates gradients (the
// optimizer step zeroes them) instead of zeroing them on entry; the LoRA
// adapters (Q and V) run inside forward / backward, so lora_forward_all /
// lora_backward_all have nothing left to do; generate() (inference) is not
// part of this library and throws RBK_ERR_UNSUPPORTED.
#pragma once

#include <cuda_runtime.h>

#include <cstdio>
#include <map>
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

// LoRAConfig (src/lora.h:13-20).  `dropout` is kept for source compatibility and not
// applied: the fused adapters run without dropout (the reference's GPU adapters never
// apply it either).
struct LoRAConfig {
    int rank = 16;
    float alpha = 32.0f;
    float dropout = 0.1f;
    float scaling() const { return alpha / rank; }
};

struct RubidiumTransformer;

// The reference keeps its adapters in a global (src/lora.h:218); here they belong to a
// model, and the free functions act on the model that last called init().
struct LoRAWeights {
    RubidiumTransformer* model = nullptr;
    LoRAConfig cfg;
    int L = 0, D = 0;
    bool initialized = false;
    // adapter parameters: A [D, r] and B [r, D] for Q and V in every layer
    long long count_params() const { return initialized ? 4LL * L * D * cfg.rank : 0; }
};

inline RubidiumTransformer*& bound_model() {
    static RubidiumTransformer* m = nullptr;
    return m;
}
inline LoRAWeights g_lora;   // src/lora.h:218

struct RubidiumTransformer {
    ModelConfig cfg;
    rbk_model* handle = nullptr;
    cudaStream_t stream = nullptr;     // the reference runs on the legacy default stream
    float loss_scale = 65536.0f;       // mirrors the device scaler (src/model.h:120)
    bool overflow = false;             // last step skipped (src/model.h:121)
    int applied_steps = 0;             // optimizer updates applied (device scaler)
    float pending_clip = 0.0f;
    std::map<unsigned char, int> char_to_id;   // src/model.h:116-117, stored in the checkpoint
    std::map<int, unsigned char> id_to_char;
    uint64_t seed = 42;                // init_weights seed (src/model.cu:146: mt19937(42))
    int max_batch = 0;                 // sequences of cfg.T tokens the activations hold
    bool configured = false;

    // init (src/model.h:122): keeps the config and binds the LoRA free functions to this
    // model; device memory is allocated by allocate_activations or at first use.
    void init(const ModelConfig& c) {
        free_all();
        cfg = c;
        configured = true;
        bound_model() = this;
    }
    // One-call form: init + allocate for max_batch sequences, weights from `seed`.
    void init(const ModelConfig& c, int max_batch_seqs, uint64_t init_seed = 42) {
        init(c);
        seed = init_seed;
        allocate_activations(max_batch_seqs * c.T);
    }
    // allocate_activations (src/model.h:125): activations for max_BT tokens, i.e.
    // ceil(max_BT / T) sequences of cfg.T.  Allocates the model on the first call.
    void allocate_activations(int max_BT) {
        if (!configured) throw Error(RBK_ERR_INVALID, "allocate_activations before init");
        const int want = (max_BT + cfg.T - 1) / cfg.T;
        if (handle) {
            if (want > max_batch)
                throw Error(RBK_ERR_INVALID, "allocate_activations: the model is already allocated for " +
                                                 std::to_string(max_batch) + " sequences");
            return;
        }
        create(want < 1 ? 1 : want);
        check(rbk_model_init_weights(handle, seed, 0.02f, stream), "rbk_model_init_weights");
    }
    void free_activations() {}         // freed with the model (free_all)
    void allocate_weights() { ensure(); }
    void init_weights() {
        ensure();
        check(rbk_model_init_weights(handle, seed, 0.02f, stream), "rbk_model_init_weights");
    }
    void convert_weights_fp32_to_fp16() { ensure(); check(rbk_model_sync_fp16(handle, stream), "rbk_model_sync_fp16"); }

    // forward (src/model.h:130): returns the mean loss (synchronises, as the reference does).
    float forward(const int* d_tokens, const int* d_targets, int B, int T) {
        ensure();
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
        ensure();
        check(rbk_model_backward(handle, d_tokens, d_targets, B, T, loss_scale_arg, stream), "rbk_model_backward");
    }
    // clip_gradients (src/model.h:133): per-tensor L2 clip, applied inside the next optimizer_step.
    void clip_gradients(float max_norm) { pending_clip = max_norm; }
    // optimizer_step (src/model.h:132): overflow check + unscale + clip + AdamW + FP16 copy + skip.
    void optimizer_step(int t, float lr, float b1, float b2, float eps, float wd) {
        ensure();
        check(rbk_model_optimizer_step(handle, t, lr, b1, b2, eps, wd, pending_clip, stream),
              "rbk_model_optimizer_step");
        pending_clip = 0.0f;
    }
    // update_loss_scale (src/model.h:134): the tail already updated the scaler; read it back.
    void update_loss_scale(bool /*overflow*/) {
        ensure();
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
    // generate (src/model.h:135): sampling is inference, outside this training library.
    std::string generate(const std::string& /*seed*/, int /*max_chars*/, float /*temp*/ = 0.7f, int /*topk*/ = 40) {
        throw Error(RBK_ERR_UNSUPPORTED, "generate: text generation is not part of librbk (training step only)");
    }
    // save / load (src/model.h:136-137): the reference's RBN2 file plus masters, Adam moments and
    // the loss scaler (rbk_model_save / rbk_model_load).  The 256-entry character map holds
    // char_to_id (src/model.cu:595-597); load restores char_to_id / id_to_char from it with the
    // reference's rule (an entry is present when its id is non-zero or it is character 0,
    // src/model.cu:645-651).  load on a model that was never allocated takes the config from the
    // file; the activations hold max(1, pending allocate_activations) sequences of cfg.T tokens.
    void save(const char* path) {
        ensure();
        int map[256] = {};
        for (const auto& kv : char_to_id) map[kv.first] = kv.second;
        check(rbk_model_save(handle, path, map, stream), "rbk_model_save");
    }
    void load(const char* path) {
        if (!handle) {
            int hdr[7] = {};                 // magic + V T D H L FF
            FILE* f = std::fopen(path, "rb");
            const bool ok = f && std::fread(hdr, sizeof(int), 7, f) == 7;
            if (f) std::fclose(f);
            if (!ok) throw Error(RBK_ERR_IO, std::string("cannot read the header of ") + path);
            ModelConfig c = cfg;
            c.init(hdr[1], hdr[2], hdr[3], hdr[4], hdr[5], hdr[6]);
            cfg = c;
            configured = true;
            if (!bound_model()) bound_model() = this;
            create(max_batch > 0 ? max_batch : 1);
        }
        int map[256] = {};
        check(rbk_model_load(handle, path, map, stream), "rbk_model_load");
        char_to_id.clear();
        id_to_char.clear();
        for (int i = 0; i < 256; ++i) {
            if (map[i] != 0 || i == 0) {
                char_to_id[(unsigned char)i] = map[i];
                id_to_char[map[i]] = (unsigned char)i;
            }
        }
        update_loss_scale(false);
    }
    // The whole trainer loop of src/main.cpp:125-175 on the device (rbk_model_train): the token
    // stream stays resident (d_stream, n tokens), windows are drawn on the device from `seed`,
    // nothing synchronises until the per-step losses are read back at the end.
    void train(const int* d_stream, int64_t n, int steps, int GA, int BS, int max_steps, int warmup, float lr,
               float b1, float b2, float eps, float wd, float gc, float* losses, uint64_t window_seed = 1) {
        ensure();
        rbk_train_args a{};
        a.tokens = d_stream; a.n_tokens = n; a.starts = nullptr; a.seed = window_seed;
        a.steps = steps; a.ga = GA; a.B = BS; a.T = cfg.T; a.first_step = applied_steps + 1;
        a.max_steps = max_steps; a.warmup = warmup;
        a.lr = lr; a.b1 = b1; a.b2 = b2; a.eps = eps; a.wd = wd; a.clip = gc;
        a.grad_scale = 1.0f / (BS * GA);      // the reference's backward factor (src/main.cpp:158)
        a.losses = losses;
        check(rbk_model_train(handle, &a, stream), "rbk_model_train");
        update_loss_scale(false);
    }
    // Data parallel (no counterpart in the single-GPU reference): join the NCCL communicator
    // (id from rbk_dp_unique_id on rank 0, shared out of band); gradients are all-reduced in
    // bucket_bytes buckets during backward.  set_grad_sync(false) makes the following backwards
    // accumulate locally (the first GA - 1 micro-steps of a step); train() sets it itself.
    void dp_init(const void* id128, int rank, int world, long long bucket_bytes = 25LL << 20) {
        ensure();
        check(rbk_model_dp_init(handle, id128, rank, world, bucket_bytes), "rbk_model_dp_init");
    }
    void set_grad_sync(bool sync) { ensure(); check(rbk_model_dp_set_sync(handle, sync ? 1 : 0), "rbk_model_dp_set_sync"); }
    // LoRA hooks (src/lora.h:223-231) as methods; the free functions below forward here.
    void init_lora(const LoRAConfig& lc, uint64_t lora_seed = 7) {
        ensure();
        check(rbk_model_lora_enable(handle, lc.rank, lc.alpha, lora_seed, stream), "rbk_model_lora_enable");
        if (bound_model() == this) {
            g_lora.model = this;
            g_lora.cfg = lc;
            g_lora.L = cfg.L;
            g_lora.D = cfg.D;
            g_lora.initialized = true;
        }
    }
    void lora_optimizer_step(int t, float lr, float b1, float b2, float eps, float wd) {
        ensure();
        check(rbk_model_lora_step(handle, t, lr, b1, b2, eps, wd, stream), "rbk_model_lora_step");
        pending_clip = 0.0f;   // the frozen base has no update for a clip to apply to
    }
    void free_all() {
        if (handle) rbk_model_destroy(handle);
        handle = nullptr;
        max_batch = 0;
        if (g_lora.model == this) g_lora = LoRAWeights();
        if (bound_model() == this) bound_model() = nullptr;
    }
    ~RubidiumTransformer() { free_all(); }

  private:
    void create(int batch) {
        rbk_config lay{cfg.V, cfg.T, cfg.D, cfg.H, cfg.L, cfg.FF};
        rbk_model_opts o{batch, cfg.T, cfg.use_activation_checkpointing ? 1 : 0, 65536.0f, 2000, 0};
        cudaGetDevice(&o.device);
        check(rbk_model_create(&handle, &lay, &o), "rbk_model_create");
        max_batch = batch;
    }
    void ensure() {
        if (handle) return;
        if (!configured) throw Error(RBK_ERR_INVALID, "RubidiumTransformer used before init");
        allocate_activations(cfg.T);
    }
};

// ---- the reference's LoRA free functions (src/lora.h:223-231) ------------------------------
// init_lora: adapters of rank cfg.rank on the Q and V projections of the model that last called
// init (its D must equal d_model); d_ff is accepted for the signature (no FFN adapters here).
inline void init_lora(int d_model, int /*d_ff*/, const LoRAConfig& lc) {
    RubidiumTransformer* m = bound_model();
    if (!m) throw Error(RBK_ERR_INVALID, "init_lora: no RubidiumTransformer has been initialised");
    if (m->cfg.D != d_model) throw Error(RBK_ERR_INVALID, "init_lora: d_model differs from the model's D");
    m->init_lora(lc);
}
// The adapters run inside RubidiumTransformer::forward / backward (fused with the Q and V
// projections), so these two have no work left; they keep the reference's signatures
// (the cuBLAS handle arrives as an opaque pointer).
inline void lora_forward_all(const float*, float*, float*, float*, float*, float*, float*, int, void*) {}
inline void lora_backward_all(const float*, const float*, const float*, const float*, const float*, const float*,
                              const float*, int, void*) {}
inline void lora_optimizer_step(int t, float lr, float b1, float b2, float eps, float wd) {
    if (!g_lora.initialized || !g_lora.model) throw Error(RBK_ERR_INVALID, "lora_optimizer_step before init_lora");
    g_lora.model->lora_optimizer_step(t, lr, b1, b2, eps, wd);
}
// lora_free (src/lora.h:231): detaches the global adapter state; the adapter memory belongs to
// the model and is released by its free_all / destructor.
inline void lora_free() { g_lora = LoRAWeights(); }

}  // namespace rubidium
