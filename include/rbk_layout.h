/*
 * rbk_layout.h — the flat parameter arena shared by every buffer family of the
 * rubidium-train decoder (FP16 weights, FP32 masters, FP32 gradients, FP32 Adam
 * m and v).
 *
 * The reference allocates each tensor with its own cudaMalloc
 * (src/model.cu:29-82) and names them through LayerWeights / ModelWeights
 * (src/model.h:29-82).  Here every family is ONE allocation and each named
 * tensor is an offset into it, so that
 *   - the fused Adam tail runs over all parameters in one launch,
 *   - gradient buckets for the data-parallel all-reduce are contiguous slices,
 *   - wq|wk|wv form one [3D, D] matrix (and bq|bk|bv one [3D] vector), so the
 *     QKV projection and its dgrad/wgrad are single GEMMs.
 *
 * Order in the arena (element offsets, all families identical):
 *   token_emb [V,D], pos_emb [T,D],
 *   layer 0 .. L-1, each: ln1_w, ln1_b, wq, wk, wv, bq, bk, bv, wo, bo,
 *                         ln2_w, ln2_b, w1 [FF,D], b1 [FF], w2 [D,FF], b2 [D]
 *   ln_f_w, ln_f_b, lm_w [V,D], lm_b [V]
 * Backward finishes gradients from the end of the arena towards its start
 * (head first, embeddings last), which is the order the all-reduce buckets
 * are launched in.
 *
 * Weights are [out, in] row-major, as the reference GPU kernels index them
 * (src/cuda_kernels.cu:756-767 reads wq[j*D + d]; lm_w is [V, D],
 * src/model.cu:47).  Every tensor starts on a 64-element boundary.
 * Requires D % 64 == 0 and FF % 64 == 0 (wq|wk|wv and bq|bk|bv stay adjacent).
 */
#ifndef RBK_LAYOUT_H
#define RBK_LAYOUT_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ModelConfig (src/model.h:16-24): V vocab, T max positions, D model width,
 * H heads, L layers, FF feed-forward width. */
typedef struct rbk_config {
    int V, T, D, H, L, FF;
} rbk_config;

enum {
    RBK_TOK_EMB = 0, RBK_POS_EMB = 1,
    RBK_N_HEAD_GLOBALS = 2,          /* tensors before layer 0 */
    RBK_LN_F_W = 0, RBK_LN_F_B = 1, RBK_LM_W = 2, RBK_LM_B = 3,
    RBK_N_TAIL_GLOBALS = 4           /* tensors after layer L-1 */
};

enum {
    RBK_LN1_W = 0, RBK_LN1_B, RBK_WQ, RBK_WK, RBK_WV, RBK_BQ, RBK_BK, RBK_BV,
    RBK_WO, RBK_BO, RBK_LN2_W, RBK_LN2_B, RBK_W1, RBK_B1, RBK_W2, RBK_B2,
    RBK_N_LAYER_TENSORS
};

typedef struct rbk_tensor {
    int64_t offset;   /* element offset into the arena */
    int64_t rows;     /* [rows, cols] row-major; vectors have rows == 1 */
    int64_t cols;
} rbk_tensor;

#define RBK_ALIGN_ELEMS 64

static inline int64_t rbk__round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

static inline int rbk_num_tensors(const rbk_config* c) {
    return RBK_N_HEAD_GLOBALS + RBK_N_LAYER_TENSORS * c->L + RBK_N_TAIL_GLOBALS;
}

/* Shape of tensor `idx` (arena order). */
static inline void rbk__shape(const rbk_config* c, int idx, int64_t* r, int64_t* k) {
    const int64_t V = c->V, T = c->T, D = c->D, F = c->FF;
    const int nl = RBK_N_LAYER_TENSORS * c->L;
    if (idx == RBK_TOK_EMB) { *r = V; *k = D; return; }
    if (idx == RBK_POS_EMB) { *r = T; *k = D; return; }
    if (idx < RBK_N_HEAD_GLOBALS + nl) {
        int j = (idx - RBK_N_HEAD_GLOBALS) % RBK_N_LAYER_TENSORS;
        switch (j) {
            case RBK_WQ: case RBK_WK: case RBK_WV: case RBK_WO: *r = D; *k = D; return;
            case RBK_W1: *r = F; *k = D; return;
            case RBK_W2: *r = D; *k = F; return;
            case RBK_B1: *r = 1; *k = F; return;
            default: *r = 1; *k = D; return;
        }
    }
    switch (idx - RBK_N_HEAD_GLOBALS - nl) {
        case RBK_LN_F_W: case RBK_LN_F_B: *r = 1; *k = D; return;
        case RBK_LM_W: *r = V; *k = D; return;
        default: *r = 1; *k = V; return;
    }
}

/* Fill `out[0 .. rbk_num_tensors)` and return the arena size in elements. */
static inline int64_t rbk_param_table(const rbk_config* c, rbk_tensor* out) {
    int64_t off = 0;
    const int n = rbk_num_tensors(c);
    for (int i = 0; i < n; ++i) {
        int64_t r, k;
        rbk__shape(c, i, &r, &k);
        if (out) { out[i].offset = off; out[i].rows = r; out[i].cols = k; }
        off += rbk__round_up(r * k, RBK_ALIGN_ELEMS);
    }
    return off;
}

static inline int64_t rbk_num_params(const rbk_config* c) { return rbk_param_table(c, 0); }

/* Arena index of layer tensor j of layer l, and of the tail globals. */
static inline int rbk_layer_tensor(int l, int j) { return RBK_N_HEAD_GLOBALS + RBK_N_LAYER_TENSORS * l + j; }
static inline int rbk_tail_tensor(const rbk_config* c, int j) {
    return RBK_N_HEAD_GLOBALS + RBK_N_LAYER_TENSORS * c->L + j;
}

/* 0 when the configuration can be laid out, else a negative code. */
static inline int rbk_config_check(const rbk_config* c) {
    if (c->V <= 0 || c->T <= 0 || c->D <= 0 || c->H <= 0 || c->L <= 0 || c->FF <= 0) return -1;
    if (c->D % 64 || c->FF % 64) return -2;
    if (c->D % c->H) return -3;
    if ((c->D / c->H) != 64 && (c->D / c->H) != 128) return -4;   /* attention: d_head 64 or 128 */
    return 0;
}

#ifdef __cplusplus
}
#endif
#endif /* RBK_LAYOUT_H */
