// model.h — host-side model state of librbk: the RubidiumTransformer drop-in.
//
// Field names follow the reference's src/model.h:16-139 (ModelConfig,
// LayerWeights, ModelWeights, Activations::LayerActs, RubidiumTransformer) so
// code written against that header reads the same; every weight / master /
// gradient / moment pointer is an offset into one arena per family
// (include/rbk_layout.h), which is what makes the fused Adam tail and the
// bucketed all-reduce single operations.
#pragma once

#include <nccl.h>

#include <vector>

#include "common.cuh"

namespace rbk {

struct ModelConfig {   // src/model.h:16-24
    int V, T, D, H, L, FF, hd;
    bool use_fp16 = true;
    bool use_activation_checkpointing = true;
    int grad_accum_steps = 1;
};

struct LayerWeights {  // src/model.h:29-55
    half *ln1_w, *ln1_b, *ln2_w, *ln2_b;
    half *wq, *bq, *wk, *bk, *wv, *bv, *wo, *bo;
    half *w1, *b1, *w2, *b2;
    float *ln1_w_fp32, *ln1_b_fp32, *ln2_w_fp32, *ln2_b_fp32;
    float *wq_fp32, *bq_fp32, *wk_fp32, *bk_fp32, *wv_fp32, *bv_fp32, *wo_fp32, *bo_fp32;
    float *w1_fp32, *b1_fp32, *w2_fp32, *b2_fp32;
    float *g_ln1_w, *g_ln1_b, *g_ln2_w, *g_ln2_b;
    float *g_wq, *g_bq, *g_wk, *g_bk, *g_wv, *g_bv, *g_wo, *g_bo;
    float *g_w1, *g_b1, *g_w2, *g_b2;
};

struct ModelWeights {  // src/model.h:60-82
    half *token_emb, *pos_emb, *ln_f_w, *ln_f_b, *lm_w, *lm_b;
    float *token_emb_fp32, *pos_emb_fp32, *ln_f_w_fp32, *ln_f_b_fp32, *lm_w_fp32, *lm_b_fp32;
    float *g_token_emb, *g_pos_emb, *g_ln_f_w, *g_ln_f_b, *g_lm_w, *g_lm_b;
    std::vector<LayerWeights> layers;
};

// Activations (src/model.h:87-107).  With checkpointing only the reference's
// recompute points are kept per layer: the layer input x (the previous
// layer's output), x1_checkpoint (post-attention residual) and h2_checkpoint
// (LN2 output), plus LN statistics; h1, q|k|v, attention output/LSE, the FFN
// pre-activation and activation live in per-model scratch and are recomputed
// in the backward.
struct LayerActs {
    half *x_in;                     // layer input [N, D]
    half *x1_checkpoint;            // [N, D]
    half *h2_checkpoint;            // [N, D]
    float *ln1_mean, *ln1_inv_std, *ln2_mean, *ln2_inv_std;
    // only without checkpointing (else point at the shared scratch)
    half *h1, *qkv, *ao, *fi_pre, *fi;
    float* lse;
};

struct Activations {
    std::vector<LayerActs> layers;
    half* x_out;                    // output of the last layer [N, D]
    half *hf, *logits;              // [N, D], [N, ldV] (dlogits in place)
    float *ln_f_mean, *ln_f_inv_std, *row_loss;
    // shared scratch (recompute targets / backward temporaries)
    half *s_h1, *s_qkv, *s_ao, *s_pre, *s_fi;
    float* s_lse;
    half *g0, *g1, *dh, *dpre, *dqkv, *dao;
    float* sink;                    // [2D] discarded LN gradients of a frozen base
};

struct LoraState {
    int rank = 0;
    float alpha = 0.0f, scaling = 0.0f;
    // FP32 masters / grads / moments, layout Aq [L,D,r] | Bq [L,r,D] | Av [L,D,r] | Bv [L,r,D]
    float *p32 = nullptr, *grad = nullptr, *m = nullptr, *v = nullptr;
    half* p16 = nullptr;            // FP16 copies used by the GEMMs
    int64_t n = 0;
    half *xa = nullptr;             // [L][2][N, r] projections h1 A (saved for backward)
    half *dyb = nullptr;            // [N, r] scratch
};

// One gradient all-reduce: fired after backward unit `unit` (0 = head,
// 1..L = layers L-1..0, L+1 = embeddings), covering arena [begin, end).
struct DpBucket {
    int unit;
    int64_t begin, end;
};

struct DpWatch;   // the communicators' watchdog (dp.cu)

struct DpState {
    bool on = false;
    // false: backward only accumulates this rank's gradients (the micro-steps of a gradient
    // accumulation group before its last); true: buckets are all-reduced as they finish.
    bool sync = true;
    int rank = 0, world = 1;
    cudaStream_t stream = nullptr;
    int64_t bucket_elems = 0;
    std::vector<DpBucket> plan;
    std::vector<cudaEvent_t> layer_done;   // recorded after each layer's grads are final
    cudaEvent_t head_done = nullptr, all_done = nullptr;
    int max_ctas = 0;                      // NCCL CTA cap of the overlapped buckets (0: NCCL's default)
    DpWatch* watch = nullptr;              // owns the communicators
    // Sharded optimizer: buckets reduce-scattered, this rank updates `own` ([begin, end) pairs,
    // ascending: slice `rank` of every bucket), FP16 weights all-gathered per bucket.
    bool shard = false;
    std::vector<int64_t> own;
    float* xbuf = nullptr;                 // [1 + segments] overflow flag + clip sums, summed over ranks
    std::vector<int> unit_bucket;          // backward unit -> index into plan
    std::vector<cudaEvent_t> weights_ready;// per bucket: its FP16 all-gather finished
    cudaEvent_t tail_done = nullptr;
    bool ag_pending = false;               // all-gathers enqueued that no forward has waited for yet
    bool masters_partial = false;          // p32 / m / v hold this rank's slices only
};

}  // namespace rbk

struct rbk_model;

namespace rbk {
// dp.cu
std::vector<DpBucket> dp_plan(const rbk_config* c, int64_t bucket_elems);
int dp_unit_done(rbk_model* m, int unit, cudaStream_t st);
int dp_reduce_all(rbk_model* m, float* buf, int64_t n, cudaStream_t st);
int dp_status(rbk_model* m);
int dp_optimizer_step(rbk_model* m, const rbk_tail_args* a, cudaStream_t st);
int dp_wait_weights(rbk_model* m, int unit, cudaStream_t st);   // unit -1: every bucket
int dp_gather_state(rbk_model* m, cudaStream_t st);
// adam.cu: one optimizer-tail launch over `own` ([begin, end) pairs; empty: the whole arena),
// phases 3 (fused) or 1 / 2 (sharded, with the exchange buffer xbuf).
int tail_launch(rbk_ctx* ctx, const rbk_tail_args* a, const std::vector<int64_t>& own, int phases, float* xbuf,
                cudaStream_t st);
}  // namespace rbk

struct rbk_model {
    rbk::ModelConfig cfg;
    rbk_config lay;
    rbk_model_opts opts;
    rbk_ctx* ctx = nullptr;
    std::vector<rbk_tensor> tab;
    int64_t n = 0;
    half* p16 = nullptr;
    float *p32 = nullptr, *grad = nullptr, *m = nullptr, *v = nullptr;
    rbk_scaler* scaler = nullptr;
    float* loss_dev = nullptr;
    int ldV = 0;
    rbk::ModelWeights w;
    rbk::Activations act;
    rbk::LoraState lora;
    rbk::DpState dp;
    std::vector<int64_t> seg_off, seg_len;
    int64_t inject_offset = 0, inject_stride = 0;
    bool inject_pending = false;
    bool fused_ce = true;           // forward writes dlogits in place (training mode)
    bool dlogits_ready = false;     // set by a training-mode forward, consumed by backward
    // The gradient arena holds zeros (after creation, rbk_model_init_weights, rbk_model_zero_grad
    // or an optimizer step, which zeroes it): the next backward's weight-gradient GEMMs store
    // their single-split tiles instead of reading and adding.  Cleared by a backward that writes
    // base gradients.
    bool grads_zero = true;
    std::vector<void*> allocs;
};
