// model.cu — RubidiumTransformer drop-in: forward, backward with per-layer
// activation checkpointing, fused optimizer tail, LoRA adapters and the
// data-parallel gradient all-reduce, all driving librbk's sm_100a kernels.
//
// Reference behaviour kept (src/model.cu): weight layout [out, in], pre-LN
// blocks (:251-304), checkpoint points x1 / h2 and the layer input
// (:292-299, :383, :400-401), CE over the LM head (:311-314), dynamic loss
// scale starting at 65536 with growth interval 2000 (src/model.h:120,
// src/cuda_kernels.cu:102-116), backward's upstream multiplier argument
// (:321-350).  Changed on purpose: GELU FFN, exact LayerNorm gradient, real
// attention / FFN / bias / pos_emb gradients, gradients accumulate across
// backward calls (the reference zeroes them at the start of every backward,
// :325-340, which defeats its own gradient accumulation) and are zeroed by
// the optimizer tail.
#include <cmath>
#include <cstring>

#include "model.h"

using namespace rbk;

namespace rbk {
namespace {

int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

template <class T>
int dalloc(rbk_model* m, T** p, size_t elems) {
    void* q = nullptr;
    RBK_CUDA(cudaMalloc(&q, std::max<size_t>(elems, 1) * sizeof(T)));
    m->allocs.push_back(q);
    *p = reinterpret_cast<T*>(q);
    return RBK_OK;
}

__global__ void cast_f32_f16_kernel(half* __restrict__ dst, const float* __restrict__ src, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __float2half_rn(src[i]);
}

// Counter-based N(0, std) init (splitmix64 hash + Box-Muller): every element
// depends only on (seed, index), so any device / grid gives the same weights.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
__global__ void randn_kernel(float* __restrict__ p, int64_t n, uint64_t seed, float std) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t h = mix64(seed ^ mix64((uint64_t)i));
        const float u1 = ((h >> 40) + 1) * (1.0f / 16777217.0f);          // (0, 1]
        const float u2 = ((h >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);   // [0, 1)
        p[i] = std * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    }
}
__global__ void fill_kernel(float* __restrict__ p, int64_t n, float v) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        p[i] = v;
}
__global__ void inject_inf_kernel(half* __restrict__ d, int N, int V, int ld, int64_t offset, int64_t stride) {
    const int64_t total = (int64_t)N * V;
    const int64_t cnt = offset < total ? (total - offset + stride - 1) / stride : 0;
    for (int64_t k = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; k < cnt; k += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = offset + k * stride;
        d[(i / V) * ld + (i % V)] = __float2half(INFINITY);
    }
}

int grid_for(int64_t n, int sms) {
    int64_t g = (n + 255) / 256;
    return (int)std::min<int64_t>(std::max<int64_t>(g, 1), (int64_t)sms * 16);
}

// ---------------------------------------------------------------- GEMMs ----
// Tags the GEMMs issued in its scope for the profiler's forward / dgrad / wgrad split.
struct Role {
    rbk_ctx* ctx;
    int saved;
    Role(rbk_ctx* c, int r) : ctx(c), saved(c->gemm_role) { c->gemm_role = r; }
    ~Role() { ctx->gemm_role = saved; }
};
enum { kFwd = 0, kDgrad = 1, kWgrad = 2 };
// The destination of the GEMMs in scope is known to hold zeros.
struct CZero {
    rbk_ctx* ctx;
    int saved;
    CZero(rbk_ctx* c, bool z) : ctx(c), saved(c->gemm_c_zero) { c->gemm_c_zero = z ? 1 : 0; }
    ~CZero() { ctx->gemm_c_zero = saved; }
};

struct G {
    rbk_ctx* ctx;
    cudaStream_t st;
    int raw(int M, int N, int K, const void* A, int lda, int am, const void* B, int ldb, int bm, void* C, int ldc,
            int epi, const void* bias = nullptr, const void* aux = nullptr, int ld_aux = 0, void* aux_out = nullptr,
            float* dbias_rows = nullptr, float alpha = 1.0f) {
        rbk_gemm_desc d = {};
        d.M = M; d.N = N; d.K = K;
        d.A = A; d.lda = lda; d.a_major = am;
        d.B = B; d.ldb = ldb; d.b_major = bm;
        d.C = C; d.ldc = ldc;
        d.epilogue = epi;
        d.bias = bias; d.aux = aux; d.ld_aux = ld_aux; d.aux_out = aux_out;
        d.dbias_rows = dbias_rows;
        d.alpha = alpha;
        return rbk_gemm(ctx, &d, st);
    }
    // Y[Nt, out] = X[Nt, in] W^T  (+bias, +residual) ; ldx/ldy row strides
    int fwd(half* Y, int ldy, const half* X, int ldx, const half* W, int Nt, int in, int out, const half* bias,
            const half* res = nullptr, int ldres = 0) {
        Role r(ctx, kFwd);
        return raw(Nt, out, in, X, ldx, 0, W, in, 0, Y, ldy, RBK_EPI_STORE_F16, bias, res, ldres);
    }
    // dX[Nt, in] = dY[Nt, out] W   (optionally * gelu'(pre))
    int dgrad(half* dX, int lddx, const half* dY, int lddy, const half* W, int Nt, int in, int out,
              const half* gelu_pre = nullptr) {
        Role r(ctx, kDgrad);
        return raw(Nt, in, out, dY, lddy, 0, W, in, 1, dX, lddx, gelu_pre ? RBK_EPI_GELU_BWD : RBK_EPI_STORE_F16,
                   nullptr, gelu_pre, gelu_pre ? lddx : 0);
    }
    // dW[out, in] += dY^T X ; dbias[out] += colsum(dY)
    int wgrad(float* dW, float* dbias, const half* dY, int lddy, const half* X, int ldx, int Nt, int in, int out) {
        Role r(ctx, kWgrad);
        CZero z(ctx, c_zero);
        return raw(out, in, Nt, dY, lddy, 1, X, ldx, 1, dW, in, RBK_EPI_ACC_F32, nullptr, nullptr, 0, nullptr, dbias);
    }
    bool c_zero = false;   // the weight gradients are known to hold zeros (each is written once per backward)
};

}  // namespace

// ------------------------------------------------------------- structure ----
static void bind_pointers(rbk_model* m) {
    const int L = m->cfg.L;
    auto P16 = [&](int i) { return m->p16 + m->tab[i].offset; };
    auto P32 = [&](int i) { return m->p32 + m->tab[i].offset; };
    auto GR = [&](int i) { return m->grad + m->tab[i].offset; };
    ModelWeights& w = m->w;
    const int ltf = rbk_tail_tensor(&m->lay, 0);
    w.token_emb = P16(RBK_TOK_EMB); w.token_emb_fp32 = P32(RBK_TOK_EMB); w.g_token_emb = GR(RBK_TOK_EMB);
    w.pos_emb = P16(RBK_POS_EMB); w.pos_emb_fp32 = P32(RBK_POS_EMB); w.g_pos_emb = GR(RBK_POS_EMB);
    w.ln_f_w = P16(ltf + RBK_LN_F_W); w.ln_f_w_fp32 = P32(ltf + RBK_LN_F_W); w.g_ln_f_w = GR(ltf + RBK_LN_F_W);
    w.ln_f_b = P16(ltf + RBK_LN_F_B); w.ln_f_b_fp32 = P32(ltf + RBK_LN_F_B); w.g_ln_f_b = GR(ltf + RBK_LN_F_B);
    w.lm_w = P16(ltf + RBK_LM_W); w.lm_w_fp32 = P32(ltf + RBK_LM_W); w.g_lm_w = GR(ltf + RBK_LM_W);
    w.lm_b = P16(ltf + RBK_LM_B); w.lm_b_fp32 = P32(ltf + RBK_LM_B); w.g_lm_b = GR(ltf + RBK_LM_B);
    w.layers.resize(L);
    for (int l = 0; l < L; ++l) {
        LayerWeights& y = w.layers[l];
#define RBK_BIND(field, idx)                                  \
    y.field = P16(rbk_layer_tensor(l, idx));                  \
    y.field##_fp32 = P32(rbk_layer_tensor(l, idx));           \
    y.g_##field = GR(rbk_layer_tensor(l, idx));
        RBK_BIND(ln1_w, RBK_LN1_W) RBK_BIND(ln1_b, RBK_LN1_B) RBK_BIND(ln2_w, RBK_LN2_W) RBK_BIND(ln2_b, RBK_LN2_B)
        RBK_BIND(wq, RBK_WQ) RBK_BIND(wk, RBK_WK) RBK_BIND(wv, RBK_WV) RBK_BIND(wo, RBK_WO)
        RBK_BIND(bq, RBK_BQ) RBK_BIND(bk, RBK_BK) RBK_BIND(bv, RBK_BV) RBK_BIND(bo, RBK_BO)
        RBK_BIND(w1, RBK_W1) RBK_BIND(b1, RBK_B1) RBK_BIND(w2, RBK_W2) RBK_BIND(b2, RBK_B2)
#undef RBK_BIND
    }
}

static int allocate_activations(rbk_model* m) {
    const int N = m->opts.max_batch * m->opts.max_seq;
    const int D = m->cfg.D, F = m->cfg.FF, L = m->cfg.L, H = m->cfg.H;
    const bool ckpt = m->cfg.use_activation_checkpointing;
    Activations& a = m->act;
    a.layers.resize(L);
    RBK_TRY(dalloc(m, &a.s_h1, (size_t)N * D));
    RBK_TRY(dalloc(m, &a.s_qkv, (size_t)N * 3 * D));
    RBK_TRY(dalloc(m, &a.s_ao, (size_t)N * D));
    RBK_TRY(dalloc(m, &a.s_pre, (size_t)N * F));
    RBK_TRY(dalloc(m, &a.s_fi, (size_t)N * F));
    RBK_TRY(dalloc(m, &a.s_lse, (size_t)m->opts.max_batch * H * m->opts.max_seq));
    for (int l = 0; l < L; ++l) {
        LayerActs& la = a.layers[l];
        RBK_TRY(dalloc(m, &la.x_in, (size_t)N * D));
        RBK_TRY(dalloc(m, &la.x1_checkpoint, (size_t)N * D));
        RBK_TRY(dalloc(m, &la.h2_checkpoint, (size_t)N * D));
        RBK_TRY(dalloc(m, &la.ln1_mean, N));
        RBK_TRY(dalloc(m, &la.ln1_inv_std, N));
        RBK_TRY(dalloc(m, &la.ln2_mean, N));
        RBK_TRY(dalloc(m, &la.ln2_inv_std, N));
        if (ckpt) {
            la.h1 = a.s_h1; la.qkv = a.s_qkv; la.ao = a.s_ao; la.fi_pre = a.s_pre; la.fi = a.s_fi; la.lse = a.s_lse;
        } else {
            RBK_TRY(dalloc(m, &la.h1, (size_t)N * D));
            RBK_TRY(dalloc(m, &la.qkv, (size_t)N * 3 * D));
            RBK_TRY(dalloc(m, &la.ao, (size_t)N * D));
            RBK_TRY(dalloc(m, &la.fi_pre, (size_t)N * F));
            RBK_TRY(dalloc(m, &la.fi, (size_t)N * F));
            RBK_TRY(dalloc(m, &la.lse, (size_t)m->opts.max_batch * H * m->opts.max_seq));
        }
    }
    RBK_TRY(dalloc(m, &a.x_out, (size_t)N * D));
    RBK_TRY(dalloc(m, &a.hf, (size_t)N * D));
    RBK_TRY(dalloc(m, &a.logits, (size_t)N * m->ldV));
    RBK_TRY(dalloc(m, &a.ln_f_mean, N));
    RBK_TRY(dalloc(m, &a.ln_f_inv_std, N));
    RBK_TRY(dalloc(m, &a.row_loss, N));
    RBK_TRY(dalloc(m, &a.g0, (size_t)N * D));
    RBK_TRY(dalloc(m, &a.g1, (size_t)N * D));
    RBK_TRY(dalloc(m, &a.dh, (size_t)N * D));
    RBK_TRY(dalloc(m, &a.dpre, (size_t)N * F));
    RBK_TRY(dalloc(m, &a.dqkv, (size_t)N * 3 * D));
    RBK_TRY(dalloc(m, &a.dao, (size_t)N * D));
    RBK_TRY(dalloc(m, &a.sink, (size_t)2 * D));
    return RBK_OK;
}

// ------------------------------------------------------------- forward -----
// Recompute-able part of layer l: h1, q|k|v (+LoRA), attention -> la.h1/qkv/ao/lse.
static int layer_attn_inputs(rbk_model* m, int l, int B, int S, cudaStream_t st) {
    const int N = B * S, D = m->cfg.D, H = m->cfg.H;
    LayerWeights& y = m->w.layers[l];
    LayerActs& la = m->act.layers[l];
    G g{m->ctx, st};
    Role role(m->ctx, kFwd);
    // (in the backward's recompute this rewrites bit-identical statistics)
    RBK_TRY(rbk_ln_fwd(m->ctx, la.h1, la.ln1_mean, la.ln1_inv_std, la.x_in, y.ln1_w, y.ln1_b, N, D, 1e-5f, st));
    RBK_TRY(g.fwd(la.qkv, 3 * D, la.h1, D, y.wq, N, D, 3 * D, y.bq));
    if (m->lora.rank > 0) {
        LoraState& lo = m->lora;
        const int r = lo.rank;
        const int64_t szA = (int64_t)m->cfg.L * D * r;
        for (int t = 0; t < 2; ++t) {
            const half* Al = lo.p16 + (t ? 2 * szA : 0) + (int64_t)l * D * r;
            const half* Bl = lo.p16 + (t ? 3 * szA : szA) + (int64_t)l * r * D;
            half* xa = lo.xa + (int64_t)t * N * r;
            // xa = h1 A;  q|v += scaling * xa B, in place in the fused qkv rows
            half* col = la.qkv + (t ? 2 * D : 0);
            RBK_TRY(rbk_lora_fwd(m->ctx, col, 3 * D, xa, la.h1, D, Al, Bl, N, D, r, D, lo.scaling, st));
        }
    }
    RBK_TRY(rbk_attn_fwd(m->ctx, la.ao, la.lse, la.qkv, B, S, H, m->cfg.hd, 1.0f / sqrtf((float)m->cfg.hd), st));
    return RBK_OK;
}

// fi = gelu(h2 W1^T + b1), and the pre-activation when the backward will read it (with
// checkpointing, the forward's pre-activation is dead: the backward recomputes both)
static int layer_ffn_inputs(rbk_model* m, int l, int N, cudaStream_t st, bool store_pre) {
    const int D = m->cfg.D, F = m->cfg.FF;
    LayerWeights& y = m->w.layers[l];
    LayerActs& la = m->act.layers[l];
    G g{m->ctx, st};
    Role role(m->ctx, kFwd);
    return g.raw(N, F, D, la.h2_checkpoint, D, 0, y.w1, D, 0, store_pre ? la.fi_pre : nullptr, F, RBK_EPI_BIAS_GELU,
                 y.b1, nullptr, F, la.fi);
}

static int forward(rbk_model* m, const int* tokens, const int* targets, int B, int S, float* loss_dev,
                   cudaStream_t st) {
    const int N = B * S, D = m->cfg.D, F = m->cfg.FF, L = m->cfg.L, V = m->cfg.V;
    G g{m->ctx, st};
    // After a sharded optimizer step each unit waits for the all-gather of its FP16 weights.
    RBK_TRY(dp_wait_weights(m, L + 1, st));
    RBK_TRY(rbk_embed_fwd(m->ctx, m->act.layers[0].x_in, m->w.token_emb, m->w.pos_emb, tokens, B, S, D, V, st));
    for (int l = 0; l < L; ++l) {
        LayerWeights& y = m->w.layers[l];
        LayerActs& la = m->act.layers[l];
        RBK_TRY(dp_wait_weights(m, L - l, st));
        RBK_TRY(layer_attn_inputs(m, l, B, S, st));
        // x1 = x + ao Wo^T + bo
        RBK_TRY(g.fwd(la.x1_checkpoint, D, la.ao, D, y.wo, N, D, D, y.bo, la.x_in, D));
        RBK_TRY(rbk_ln_fwd(m->ctx, la.h2_checkpoint, la.ln2_mean, la.ln2_inv_std, la.x1_checkpoint, y.ln2_w, y.ln2_b,
                           N, D, 1e-5f, st));
        RBK_TRY(layer_ffn_inputs(m, l, N, st, !m->cfg.use_activation_checkpointing));
        half* out = (l + 1 < L) ? m->act.layers[l + 1].x_in : m->act.x_out;
        RBK_TRY(g.fwd(out, D, la.fi, F, y.w2, N, F, D, y.b2, la.x1_checkpoint, D));
    }
    RBK_TRY(dp_wait_weights(m, 0, st));
    RBK_TRY(rbk_ln_fwd(m->ctx, m->act.hf, m->act.ln_f_mean, m->act.ln_f_inv_std, m->act.x_out, m->w.ln_f_w,
                       m->w.ln_f_b, N, D, 1e-5f, st));
    RBK_TRY(g.fwd(m->act.logits, m->ldV, m->act.hf, D, m->w.lm_w, N, D, V, m->w.lm_b));
    m->dlogits_ready = false;
    if (targets) {
        // Training mode: the same pass that produces the loss writes dlogits over
        // the logits (without backward's upstream factor, applied later as the
        // LM-head GEMMs' alpha), saving a second read of [N, V].
        const float world = m->dp.on ? (float)m->dp.world : 1.0f;
        const bool fuse = m->fused_ce;
        RBK_TRY(rbk_softmax_xent_bwd(m->ctx, fuse ? m->act.logits : nullptr, m->act.logits, m->ldV, targets, N, V,
                                     1.0f / (N * world), fuse ? &m->scaler->scale : nullptr, m->act.row_loss, st));
        RBK_TRY(rbk_sum(m->ctx, loss_dev ? loss_dev : m->loss_dev, m->act.row_loss, N, 1.0f / N, st));
        m->dlogits_ready = fuse;
    }
    return RBK_OK;
}


// ------------------------------------------------------------- backward ----
static int backward(rbk_model* m, const int* tokens, const int* targets, int B, int S, float grad_scale,
                    cudaStream_t st) {
    const int N = B * S, D = m->cfg.D, F = m->cfg.FF, L = m->cfg.L, V = m->cfg.V, H = m->cfg.H;
    const bool ckpt = m->cfg.use_activation_checkpointing;
    const bool base = m->lora.rank == 0;          // frozen base under LoRA
    G g{m->ctx, st};
    Activations& a = m->act;
    const float world = m->dp.on ? (float)m->dp.world : 1.0f;
    // Gradients accumulate across backward calls; only the last micro-step of an accumulation
    // group all-reduces, so each rank's earlier micro-steps enter the sum exactly once.
    // Under LoRA the frozen base has no gradients to exchange: the adapter arena is reduced once
    // at the end instead (a few MB).
    const bool reduce = m->dp.on && m->dp.sync && m->lora.rank == 0;
    const bool reduce_lora = m->dp.on && m->dp.sync && m->lora.rank > 0;
    // dlogits = (softmax - onehot) * grad_scale / (N * world) * loss_scale, in place.  When the
    // forward already wrote it (training mode), grad_scale rides on the LM-head GEMMs' alpha.
    float head_alpha = 1.0f;
    if (m->dlogits_ready) {
        head_alpha = grad_scale;
        m->dlogits_ready = false;
    } else {
        RBK_TRY(rbk_softmax_xent_bwd(m->ctx, a.logits, a.logits, m->ldV, targets, N, V, grad_scale / (N * world),
                                     &m->scaler->scale, nullptr, st));
    }
    if (m->inject_pending) {
        inject_inf_kernel<<<grid_for((int64_t)N * V / std::max<int64_t>(m->inject_stride, 1), m->ctx->num_sms), 256,
                            0, st>>>(a.logits, N, V, m->ldV, m->inject_offset, m->inject_stride);
        RBK_LAUNCHED("inject_inf_kernel");
        m->inject_pending = false;
    }
    // LM head
    {
        Role role(m->ctx, kDgrad);
        RBK_TRY(g.raw(N, D, V, a.logits, m->ldV, 0, m->w.lm_w, D, 1, a.dh, D, RBK_EPI_STORE_F16, nullptr, nullptr, 0,
                      nullptr, nullptr, head_alpha));
    }
    // Each weight gradient is written by one GEMM per backward: right after an optimizer step (or
    // zeroing) its tiles are stored instead of read and added.
    g.c_zero = base && m->grads_zero;
    if (base) {
        Role role(m->ctx, kWgrad);
        CZero z(m->ctx, g.c_zero);
        RBK_TRY(g.raw(V, D, N, a.logits, m->ldV, 1, a.hf, D, 1, m->w.g_lm_w, D, RBK_EPI_ACC_F32, nullptr, nullptr, 0,
                      nullptr, m->w.g_lm_b, head_alpha));
        m->grads_zero = false;
    }
    // final LN (under LoRA the LN parameters are frozen: their gradients go to a sink)
    float* sk = a.sink;
    half* gcur = a.g0;
    half* gnext = a.g1;
    // Bias gradients ride on the kernels that produce the bias's upstream gradient, so the W2, Wo
    // and QKV weight gradients run on N = 256 tiles without the bias-gradient MMA: b2 of a layer
    // is the column sum of the residual gradient the LayerNorm backward above it writes, bo the
    // one LN2's backward writes, and bq|bk|bv come from the attention backward.
    RBK_TRY(rbk_ln_bwd(m->ctx, gcur, base ? m->w.g_ln_f_w : sk, base ? m->w.g_ln_f_b : sk + D,
                       base ? m->w.layers[L - 1].g_b2 : nullptr, a.dh, nullptr, a.x_out, m->w.ln_f_w, a.ln_f_mean,
                       a.ln_f_inv_std, N, D, 0, st));
    if (reduce) RBK_TRY(dp_unit_done(m, 0, st));
    for (int l = L - 1; l >= 0; --l) {
        LayerWeights& y = m->w.layers[l];
        LayerActs& la = a.layers[l];
        if (ckpt) {
            RBK_TRY(layer_attn_inputs(m, l, B, S, st));
            RBK_TRY(layer_ffn_inputs(m, l, N, st, true));
        } else if (m->lora.rank > 0) {
            // LoRA projections are recomputed from the stored h1 (they are not kept)
            RBK_TRY(layer_attn_inputs(m, l, B, S, st));
        }
        // ---- FFN: x_out = x1 + gelu(h2 W1^T + b1) W2^T + b2 ----
        if (base) RBK_TRY(g.wgrad(y.g_w2, nullptr, gcur, D, la.fi, F, N, F, D));   // b2: see above
        RBK_TRY(g.dgrad(a.dpre, F, gcur, D, y.w2, N, F, D, la.fi_pre));
        if (base) RBK_TRY(g.wgrad(y.g_w1, y.g_b1, a.dpre, F, la.h2_checkpoint, D, N, D, F));
        RBK_TRY(g.dgrad(a.dh, D, a.dpre, F, y.w1, N, D, F));
        // ---- LN2: dx1 = g + LN2'(dh) ----
        RBK_TRY(rbk_ln_bwd(m->ctx, gnext, base ? y.g_ln2_w : sk, base ? y.g_ln2_b : sk + D, base ? y.g_bo : nullptr,
                           a.dh, gcur, la.x1_checkpoint, y.ln2_w, la.ln2_mean, la.ln2_inv_std, N, D, 0, st));
        std::swap(gcur, gnext);   // gcur = dx1
        // ---- attention output projection ----
        if (base) RBK_TRY(g.wgrad(y.g_wo, nullptr, gcur, D, la.ao, D, N, D, D));   // bo: from LN2's backward
        RBK_TRY(g.dgrad(a.dao, D, gcur, D, y.wo, N, D, D));
        // ---- attention core ----
        RBK_TRY(rbk_attn_bwd(m->ctx, a.dqkv, base ? y.g_bq : nullptr, la.qkv, la.ao, a.dao, la.lse, B, S, H,
                             m->cfg.hd, 1.0f / sqrtf((float)m->cfg.hd), st));
        // ---- QKV projection (one [3D, D] GEMM each way) ----
        if (base) RBK_TRY(g.wgrad(y.g_wq, nullptr, a.dqkv, 3 * D, la.h1, D, N, D, 3 * D));   // bq|bk|bv: above
        RBK_TRY(g.dgrad(a.dh, D, a.dqkv, 3 * D, y.wq, N, D, 3 * D));
        if (m->lora.rank > 0) {
            LoraState& lo = m->lora;
            const int r = lo.rank;
            const int64_t szA = (int64_t)L * D * r;
            for (int t = 0; t < 2; ++t) {
                const half* Al = lo.p16 + (t ? 2 * szA : 0) + (int64_t)l * D * r;
                const half* Bl = lo.p16 + (t ? 3 * szA : szA) + (int64_t)l * r * D;
                float* dAl = lo.grad + (t ? 2 * szA : 0) + (int64_t)l * D * r;
                float* dBl = lo.grad + (t ? 3 * szA : szA) + (int64_t)l * r * D;
                const half* xa = lo.xa + (int64_t)t * N * r;
                const half* dy = a.dqkv + (t ? 2 * D : 0);
                // dB += s xa^T dy;  dyb = s dy B^T;  dA += h1^T dyb;  dh1 += dyb A^T
                RBK_TRY(rbk_lora_bwd(m->ctx, dAl, dBl, a.dh, D, lo.dyb, dy, 3 * D, la.h1, D, xa, Al, Bl, N, D, r, D,
                                     lo.scaling, st));
            }
        }
        // ---- LN1: g_prev = dx1 + LN1'(dh1) ----
        RBK_TRY(rbk_ln_bwd(m->ctx, gnext, base ? y.g_ln1_w : sk, base ? y.g_ln1_b : sk + D,
                           base && l > 0 ? m->w.layers[l - 1].g_b2 : nullptr, a.dh, gcur, la.x_in, y.ln1_w,
                           la.ln1_mean, la.ln1_inv_std, N, D, 0, st));
        std::swap(gcur, gnext);
        if (reduce) RBK_TRY(dp_unit_done(m, L - l, st));
    }
    if (base) RBK_TRY(rbk_embed_bwd(m->ctx, m->w.g_token_emb, m->w.g_pos_emb, gcur, tokens, B, S, D, V, st));
    if (reduce) RBK_TRY(dp_unit_done(m, L + 1, st));
    if (reduce_lora) RBK_TRY(dp_reduce_all(m, m->lora.grad, m->lora.n, st));
    return RBK_OK;
}

}  // namespace rbk

// ============================================================== C ABI =====
extern "C" {

int rbk_model_create(rbk_model** out, const rbk_config* cfg, const rbk_model_opts* opts) {
    RBK_REQUIRE(out && cfg && opts, "rbk_model_create: null pointer");
    *out = nullptr;
    const int chk = rbk_config_check(cfg);
    RBK_REQUIRE(chk == 0, "rbk_model_create: unsupported config (code %d): need D, FF %% 64 == 0, d_head 64 or 128", chk);
    RBK_REQUIRE(opts->max_batch > 0 && opts->max_seq > 0 && opts->max_seq <= cfg->T && opts->max_seq % 64 == 0,
                "rbk_model_create: need 0 < max_seq <= T and max_seq %% 64 == 0");
    rbk_model* m = new rbk_model();
    m->lay = *cfg;
    m->opts = *opts;
    m->cfg.V = cfg->V; m->cfg.T = cfg->T; m->cfg.D = cfg->D; m->cfg.H = cfg->H; m->cfg.L = cfg->L;
    m->cfg.FF = cfg->FF; m->cfg.hd = cfg->D / cfg->H;
    m->cfg.use_activation_checkpointing = opts->use_activation_checkpointing != 0;
    int st = rbk_ctx_create(&m->ctx, opts->device);
    if (st) { delete m; return st; }
    m->tab.resize(rbk_num_tensors(cfg));
    m->n = rbk_param_table(cfg, m->tab.data());
    m->ldV = (int)round_up(cfg->V, 8);
    auto fail = [&](int s) { rbk_model_destroy(m); return s; };
    if ((st = dalloc(m, &m->p16, m->n)) || (st = dalloc(m, &m->p32, m->n)) || (st = dalloc(m, &m->grad, m->n)) ||
        (st = dalloc(m, &m->m, m->n)) || (st = dalloc(m, &m->v, m->n)) || (st = dalloc(m, &m->scaler, 1)) ||
        (st = dalloc(m, &m->loss_dev, 1)))
        return fail(st);
    bind_pointers(m);
    if ((st = allocate_activations(m))) return fail(st);
    for (size_t i = 0; i < m->tab.size(); ++i) {
        m->seg_off.push_back(m->tab[i].offset);
        m->seg_len.push_back(round_up(m->tab[i].rows * m->tab[i].cols, RBK_ALIGN_ELEMS));
    }
    rbk_scaler s = {};
    s.scale = opts->init_loss_scale > 0 ? opts->init_loss_scale : 65536.0f;
    s.interval = opts->growth_interval > 0 ? opts->growth_interval : 2000;
    if (cudaMemcpy(m->scaler, &s, sizeof(s), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(m->grad, 0, sizeof(float) * m->n) != cudaSuccess ||
        cudaMemset(m->m, 0, sizeof(float) * m->n) != cudaSuccess ||
        cudaMemset(m->v, 0, sizeof(float) * m->n) != cudaSuccess ||
        cudaMemset(m->p32, 0, sizeof(float) * m->n) != cudaSuccess ||
        cudaMemset(m->p16, 0, sizeof(half) * m->n) != cudaSuccess) {
        set_error("rbk_model_create: initial copies failed");
        return fail(RBK_ERR_CUDA);
    }
    *out = m;
    return RBK_OK;
}

int rbk_model_destroy(rbk_model* m) {
    if (!m) return RBK_OK;
    if (m->ctx) cudaSetDevice(m->ctx->device);
    cudaDeviceSynchronize();
    if (m->dp.on) rbk_model_dp_shutdown(m);
    for (void* p : m->allocs) cudaFree(p);
    if (m->ctx) rbk_ctx_destroy(m->ctx);
    delete m;
    return RBK_OK;
}

int rbk_model_ctx(rbk_model* m, rbk_ctx** ctx) {
    RBK_REQUIRE(m && ctx, "rbk_model_ctx: null pointer");
    *ctx = m->ctx;
    return RBK_OK;
}

int rbk_model_buffer(rbk_model* m, int which, void** ptr, int64_t* n) {
    RBK_REQUIRE(m && ptr && n, "rbk_model_buffer: null pointer");
    *n = m->n;
    switch (which) {
        case RBK_BUF_P16: *ptr = m->p16; return RBK_OK;
        case RBK_BUF_P32: *ptr = m->p32; return RBK_OK;
        case RBK_BUF_GRAD: *ptr = m->grad; return RBK_OK;
        case RBK_BUF_M: *ptr = m->m; return RBK_OK;
        case RBK_BUF_V: *ptr = m->v; return RBK_OK;
        case RBK_BUF_LOSS: *ptr = m->loss_dev; *n = 1; return RBK_OK;
        case RBK_BUF_LOGITS:
            *ptr = m->act.logits;
            *n = (int64_t)m->opts.max_batch * m->opts.max_seq * m->ldV;
            return RBK_OK;
        default: break;
    }
    set_error("rbk_model_buffer: unknown buffer %d", which);
    return RBK_ERR_INVALID;
}

int rbk_model_scaler(rbk_model* m, rbk_scaler** dev) {
    RBK_REQUIRE(m && dev, "rbk_model_scaler: null pointer");
    *dev = m->scaler;
    return RBK_OK;
}

int rbk_model_sync_fp16(rbk_model* m, void* stream) {
    RBK_REQUIRE(m, "rbk_model_sync_fp16: null model");
    RBK_TRY(dp_gather_state(m, as_stream(stream)));   // sharded optimizer: whole masters first
    RBK_TRY(dp_wait_weights(m, -1, as_stream(stream)));
    cast_f32_f16_kernel<<<grid_for(m->n, m->ctx->num_sms), 256, 0, as_stream(stream)>>>(m->p16, m->p32, m->n);
    RBK_LAUNCHED("cast_f32_f16_kernel");
    return RBK_OK;
}

int rbk_model_init_weights(rbk_model* m, uint64_t seed, float std, void* stream) {
    RBK_REQUIRE(m, "rbk_model_init_weights: null model");
    cudaStream_t st = as_stream(stream);
    RBK_CUDA(cudaMemsetAsync(m->p32, 0, sizeof(float) * m->n, st));
    for (size_t i = 0; i < m->tab.size(); ++i) {
        const rbk_tensor& t = m->tab[i];
        const int64_t cnt = t.rows * t.cols;
        int kind;   // 0 zero, 1 one, 2 randn
        if ((int)i == RBK_TOK_EMB || (int)i == RBK_POS_EMB) kind = 2;
        else if ((int)i >= rbk_tail_tensor(&m->lay, 0)) {
            const int j = (int)i - rbk_tail_tensor(&m->lay, 0);
            kind = j == RBK_LN_F_W ? 1 : j == RBK_LM_W ? 2 : 0;
        } else {
            const int j = ((int)i - RBK_N_HEAD_GLOBALS) % RBK_N_LAYER_TENSORS;
            kind = (j == RBK_LN1_W || j == RBK_LN2_W) ? 1
                   : (j == RBK_WQ || j == RBK_WK || j == RBK_WV || j == RBK_WO || j == RBK_W1 || j == RBK_W2) ? 2 : 0;
        }
        if (kind == 1) fill_kernel<<<grid_for(cnt, m->ctx->num_sms), 256, 0, st>>>(m->p32 + t.offset, cnt, 1.0f);
        if (kind == 2)
            randn_kernel<<<grid_for(cnt, m->ctx->num_sms), 256, 0, st>>>(m->p32 + t.offset, cnt, seed * 1000003ull + i,
                                                                          std);
        RBK_LAUNCHED("init kernels");
    }
    RBK_CUDA(cudaMemsetAsync(m->grad, 0, sizeof(float) * m->n, st));
    RBK_CUDA(cudaMemsetAsync(m->m, 0, sizeof(float) * m->n, st));
    RBK_CUDA(cudaMemsetAsync(m->v, 0, sizeof(float) * m->n, st));
    m->dp.masters_partial = false;                   // every rank holds the whole state again
    m->grads_zero = true;
    return rbk_model_sync_fp16(m, stream);
}

int rbk_model_forward(rbk_model* m, const int* tokens, const int* targets, int B, int S, float* loss_dev,
                      void* stream) {
    RBK_REQUIRE(m && tokens, "rbk_model_forward: null pointer");
    RBK_REQUIRE(B > 0 && B <= m->opts.max_batch && S > 0 && S <= m->opts.max_seq && S % 64 == 0,
                "rbk_model_forward: need B <= max_batch, S <= max_seq, S %% 64 == 0 (B=%d S=%d)", B, S);
    return forward(m, tokens, targets, B, S, loss_dev, as_stream(stream));
}

int rbk_model_backward(rbk_model* m, const int* tokens, const int* targets, int B, int S, float grad_scale,
                       void* stream) {
    RBK_REQUIRE(m && tokens && targets, "rbk_model_backward: null pointer");
    if (m->dp.on) RBK_TRY(rbk_model_dp_status(m));   // an aborted communicator fails fast
    RBK_REQUIRE(B > 0 && B <= m->opts.max_batch && S > 0 && S <= m->opts.max_seq && S % 64 == 0,
                "rbk_model_backward: bad B/S");
    RBK_TRY(dp_wait_weights(m, -1, as_stream(stream)));
    return backward(m, tokens, targets, B, S, grad_scale, as_stream(stream));
}

int rbk_model_optimizer_step(rbk_model* m, int t, float lr, float b1, float b2, float eps, float wd, float max_norm,
                             void* stream) {
    RBK_REQUIRE(m, "rbk_model_optimizer_step: null model");
    if (m->dp.on) RBK_TRY(rbk_model_dp_status(m));   // never apply a partially reduced gradient
    rbk_tail_args a = {};
    a.p32 = m->p32; a.g = m->grad; a.m = m->m; a.v = m->v; a.p16 = m->p16; a.n = m->n;
    a.seg_off = m->seg_off.data(); a.seg_len = m->seg_len.data(); a.nseg = (int)m->seg_off.size();
    a.max_norm = max_norm;
    a.lr = lr; a.beta1 = b1; a.beta2 = b2; a.eps = eps; a.weight_decay = wd; a.t = t;
    a.scaler = m->scaler;
    // the tail zeroes every gradient it updates (and a sharded step the rest of each bucket)
    const int st = m->dp.on && m->dp.shard ? dp_optimizer_step(m, &a, as_stream(stream))
                                           : rbk_adam_tail(m->ctx, &a, stream);
    if (st == RBK_OK) m->grads_zero = true;
    return st;
}

int rbk_model_zero_grad(rbk_model* m, void* stream) {
    RBK_REQUIRE(m, "rbk_model_zero_grad: null model");
    RBK_CUDA(cudaMemsetAsync(m->grad, 0, sizeof(float) * m->n, as_stream(stream)));
    m->grads_zero = true;
    return RBK_OK;
}

int rbk_model_lora_enable(rbk_model* m, int rank, float alpha, uint64_t seed, void* stream) {
    RBK_REQUIRE(m && rank > 0 && rank % 8 == 0 && rank <= 64, "rbk_model_lora_enable: rank must be 8..64, %% 8 == 0");
    RBK_REQUIRE(m->lora.rank == 0, "rbk_model_lora_enable: already enabled");
    RBK_REQUIRE(!m->dp.shard, "rbk_model_lora_enable: not with the sharded optimizer (it covers the base model)");
    LoraState& lo = m->lora;
    const int64_t szA = (int64_t)m->cfg.L * m->cfg.D * rank;
    lo.n = 4 * szA;
    const int N = m->opts.max_batch * m->opts.max_seq;
    RBK_TRY(dalloc(m, &lo.p32, lo.n));
    RBK_TRY(dalloc(m, &lo.grad, lo.n));
    RBK_TRY(dalloc(m, &lo.m, lo.n));
    RBK_TRY(dalloc(m, &lo.v, lo.n));
    RBK_TRY(dalloc(m, &lo.p16, lo.n));
    RBK_TRY(dalloc(m, &lo.xa, (size_t)2 * N * rank));
    RBK_TRY(dalloc(m, &lo.dyb, (size_t)N * rank));
    cudaStream_t st = as_stream(stream);
    RBK_CUDA(cudaMemsetAsync(lo.p32, 0, sizeof(float) * lo.n, st));
    RBK_CUDA(cudaMemsetAsync(lo.grad, 0, sizeof(float) * lo.n, st));
    RBK_CUDA(cudaMemsetAsync(lo.m, 0, sizeof(float) * lo.n, st));
    RBK_CUDA(cudaMemsetAsync(lo.v, 0, sizeof(float) * lo.n, st));
    // A ~ N(0, 0.02) (cpu_lora.h:29-31), B = 0
    randn_kernel<<<grid_for(szA, m->ctx->num_sms), 256, 0, st>>>(lo.p32, szA, seed * 7919ull + 1, 0.02f);
    randn_kernel<<<grid_for(szA, m->ctx->num_sms), 256, 0, st>>>(lo.p32 + 2 * szA, szA, seed * 7919ull + 2, 0.02f);
    cast_f32_f16_kernel<<<grid_for(lo.n, m->ctx->num_sms), 256, 0, st>>>(lo.p16, lo.p32, lo.n);
    RBK_LAUNCHED("lora init");
    lo.rank = rank;
    lo.alpha = alpha;
    lo.scaling = alpha / rank;
    return RBK_OK;
}

int rbk_model_lora_buffer(rbk_model* m, int which, void** ptr, int64_t* n) {
    RBK_REQUIRE(m && ptr && n && m->lora.rank > 0, "rbk_model_lora_buffer: LoRA not enabled");
    *n = m->lora.n;
    switch (which) {
        case RBK_BUF_P16: *ptr = m->lora.p16; return RBK_OK;
        case RBK_BUF_P32: *ptr = m->lora.p32; return RBK_OK;
        case RBK_BUF_GRAD: *ptr = m->lora.grad; return RBK_OK;
        case RBK_BUF_M: *ptr = m->lora.m; return RBK_OK;
        case RBK_BUF_V: *ptr = m->lora.v; return RBK_OK;
        default: break;
    }
    set_error("rbk_model_lora_buffer: unknown buffer %d", which);
    return RBK_ERR_INVALID;
}

int rbk_model_lora_step(rbk_model* m, int t, float lr, float b1, float b2, float eps, float wd, void* stream) {
    RBK_REQUIRE(m && m->lora.rank > 0, "rbk_model_lora_step: LoRA not enabled");
    if (m->dp.on) RBK_TRY(rbk_model_dp_status(m));
    rbk_tail_args a = {};
    a.p32 = m->lora.p32; a.g = m->lora.grad; a.m = m->lora.m; a.v = m->lora.v; a.p16 = m->lora.p16;
    a.n = m->lora.n;
    a.lr = lr; a.beta1 = b1; a.beta2 = b2; a.eps = eps; a.weight_decay = wd; a.t = t;
    a.scaler = m->scaler;
    return rbk_adam_tail(m->ctx, &a, stream);
}

int rbk_model_set_training(rbk_model* m, int training) {
    RBK_REQUIRE(m, "rbk_model_set_training: null model");
    m->fused_ce = training != 0;
    m->dlogits_ready = false;
    return RBK_OK;
}

int rbk_model_inject_inf(rbk_model* m, int64_t offset, int64_t stride) {
    RBK_REQUIRE(m, "rbk_model_inject_inf: null model");
    m->inject_offset = offset;
    m->inject_stride = stride;
    m->inject_pending = stride > 0;
    return RBK_OK;
}

}  // extern "C"
