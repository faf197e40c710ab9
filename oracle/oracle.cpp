// oracle.cpp — FP32 CPU restatement of the rubidium-train training step.
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path is
// compared against: only tests/, __graft_entry__.smoke() and bench.py's CPU
// baseline leg load it.  No product code links it.
//
// What it restates, op by op (reference paths are relative to its project):
//   matmul conventions          src/cpu_mat.h:47-95
//   LayerNorm fwd / bwd         src/cpu_mat.h:98-153  (eps 1e-5, biased var)
//   softmax bwd                 src/cpu_mat.h:190-200
//   cross-entropy fwd / bwd     src/cpu_mat.h:203-236 (mean over rows, +1e-10 in the log)
//   embedding bwd               src/cpu_mat.h:265-277
//   AdamW (L2-coupled)          src/cpu_mat.h:280-292, backup/cuda_kernels.cu.bak:462-473
//   per-tensor clip             src/cpu_mat.h:295-306
//   loss scaler                 src/cuda_kernels.cu:102-116
//   attention fwd               src/cpu_model.cpp:148-180 (scale 1/sqrt(d_h), mask -1e9)
//   pre-LN block                src/cpu_model.cpp:126-207, src/model.cu:251-304
// Deviations from the reference, all deliberate and shared with the CUDA path:
//   GELU (tanh form) instead of ReLU (ReLU kept as a mode for pinning);
//   weights are [out, in] (y = x W^T), LM head h W_lm^T with W_lm [V, D];
//   batched sequences; full gradients incl. lm_b and pos_emb; attention and
//   FFN gradients are computed (the reference leaves them as placeholders).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#include <omp.h>

#include "../include/rbk_layout.h"

namespace {

// ---------------------------------------------------------------------------
// GEMM: C[M,N] = beta*C + op(A)[M,K] * op(B)[K,N]  (row-major, FP32 accumulate)
// Same arithmetic as cpuops::matmul / matmul_tB / matmul_tA (cpu_mat.h:47-95),
// cache-blocked so the CPU baseline stays usable at GPT-2-small shapes.
// ---------------------------------------------------------------------------
void gemm(int M, int N, int K, const float* A, int lda, bool tA, const float* B, int ldb, bool tB,
          float* C, int ldc, float beta) {
    // Pack op(B) into Bp[K][N] so the inner loop runs along contiguous N.
    std::vector<float> Bp((size_t)K * N);
#pragma omp parallel for schedule(static)
    for (int k = 0; k < K; ++k)
        for (int j = 0; j < N; ++j)
            Bp[(size_t)k * N + j] = tB ? B[(size_t)j * ldb + k] : B[(size_t)k * ldb + j];
    const int MB = 16, KB = 256, NB = 1024;
    const int nmb = (M + MB - 1) / MB, nnb = (N + NB - 1) / NB;
#pragma omp parallel for schedule(dynamic) collapse(2)
    for (int ib = 0; ib < nmb; ++ib) {
        for (int jb = 0; jb < nnb; ++jb) {
            const int i0 = ib * MB, i1 = std::min(M, i0 + MB);
            const int j0 = jb * NB, j1 = std::min(N, j0 + NB);
            const int nj = j1 - j0;
            float acc[MB][NB];
            for (int i = i0; i < i1; ++i)
                for (int j = 0; j < nj; ++j) acc[i - i0][j] = 0.0f;
            for (int k0 = 0; k0 < K; k0 += KB) {
                const int k1 = std::min(K, k0 + KB);
                for (int i = i0; i < i1; ++i) {
                    float* ar = acc[i - i0];
                    for (int k = k0; k < k1; ++k) {
                        const float a = tA ? A[(size_t)k * lda + i] : A[(size_t)i * lda + k];
                        const float* br = &Bp[(size_t)k * N + j0];
                        for (int j = 0; j < nj; ++j) ar[j] += a * br[j];
                    }
                }
            }
            for (int i = i0; i < i1; ++i) {
                float* cr = C + (size_t)i * ldc + j0;
                if (beta == 0.0f)
                    for (int j = 0; j < nj; ++j) cr[j] = acc[i - i0][j];
                else
                    for (int j = 0; j < nj; ++j) cr[j] = beta * cr[j] + acc[i - i0][j];
            }
        }
    }
}

// y = x W^T + b   (W [out, in])
void linear(float* y, const float* x, const float* W, const float* b, int N, int in, int out) {
    gemm(N, out, in, x, in, false, W, in, true, y, out, 0.0f);
    if (b) {
#pragma omp parallel for schedule(static)
        for (int n = 0; n < N; ++n)
            for (int j = 0; j < out; ++j) y[(size_t)n * out + j] += b[j];
    }
}

// Backward of y = x W^T + b.  dW += dy^T x, db += colsum(dy), dx = dy W (or += when accumulate).
void linear_bwd(float* dx, bool dx_accumulate, float* dW, float* db, const float* dy, const float* x,
                const float* W, int N, int in, int out) {
    if (dx) gemm(N, in, out, dy, out, false, W, in, false, dx, in, dx_accumulate ? 1.0f : 0.0f);
    if (dW) gemm(out, in, N, dy, out, true, x, in, false, dW, in, 1.0f);
    if (db) {
#pragma omp parallel for schedule(static)
        for (int j = 0; j < out; ++j) {
            float s = 0.0f;
            for (int n = 0; n < N; ++n) s += dy[(size_t)n * out + j];
            db[j] += s;
        }
    }
}

// LayerNorm forward, cpu_mat.h:98-123 (two-pass mean / biased variance).
void ln_fwd(float* y, float* mean, float* rstd, const float* x, const float* g, const float* b, int N, int D,
            float eps) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < N; ++i) {
        const float* xr = x + (size_t)i * D;
        float m = 0.0f;
        for (int j = 0; j < D; ++j) m += xr[j];
        m /= D;
        float v = 0.0f;
        for (int j = 0; j < D; ++j) { float d = xr[j] - m; v += d * d; }
        float inv = 1.0f / std::sqrt(v / D + eps);
        mean[i] = m; rstd[i] = inv;
        for (int j = 0; j < D; ++j) y[(size_t)i * D + j] = g[j] * (xr[j] - m) * inv + b[j];
    }
}

// LayerNorm backward, cpu_mat.h:126-153.  dg/db accumulate (+=); dx written, or
// added to when dx_accumulate (the residual branch).
//
// The reference computes dx = inv (g w - (ts1 + (x - m) inv ts2) / D) with
// ts2 = sum g w (x - m) (cpu_mat.h:146, same at cuda_kernels.cu:276).  The
// exact gradient needs (x - m) inv^2 ts2 in that term: the reference drops one
// factor of rstd, which only vanishes when rstd == 1.  ref_formula = true
// reproduces the reference's expression (used to pin against its engine);
// the model and the CUDA path use the exact gradient.
void ln_bwd(float* dx, bool dx_accumulate, float* dg, float* db, const float* dy, const float* x, const float* g,
            const float* mean, const float* rstd, int N, int D, bool ref_formula = false) {
    std::vector<float> pdg((size_t)omp_get_max_threads() * D, 0.0f), pdb((size_t)omp_get_max_threads() * D, 0.0f);
#pragma omp parallel
    {
        float* mydg = &pdg[(size_t)omp_get_thread_num() * D];
        float* mydb = &pdb[(size_t)omp_get_thread_num() * D];
#pragma omp for schedule(static)
        for (int i = 0; i < N; ++i) {
            const float* dyr = dy + (size_t)i * D;
            const float* xr = x + (size_t)i * D;
            const float m = mean[i], inv = rstd[i];
            float ts1 = 0.0f, ts2 = 0.0f;
            for (int j = 0; j < D; ++j) {
                float dwj = dyr[j] * g[j];
                ts1 += dwj;
                ts2 += dwj * (xr[j] - m);
            }
            for (int j = 0; j < D; ++j) {
                float dwj = dyr[j] * g[j];
                const float c2 = ref_formula ? inv : inv * inv;
                float v = inv * (dwj - (ts1 + (xr[j] - m) * c2 * ts2) / D);
                if (dx_accumulate) dx[(size_t)i * D + j] += v; else dx[(size_t)i * D + j] = v;
                mydg[j] += dyr[j] * (xr[j] - m) * inv;
                mydb[j] += dyr[j];
            }
        }
    }
    for (int t = 0; t < omp_get_max_threads(); ++t)
        for (int j = 0; j < D; ++j) { dg[j] += pdg[(size_t)t * D + j]; db[j] += pdb[(size_t)t * D + j]; }
}

const float kGeluC = 0.7978845608028654f;   // sqrt(2/pi)
const float kGeluA = 0.044715f;

inline float act_fwd(float x, int relu) {
    if (relu) return x > 0.0f ? x : 0.0f;
    float u = kGeluC * (x + kGeluA * x * x * x);
    return 0.5f * x * (1.0f + std::tanh(u));
}
inline float act_grad(float x, int relu) {
    if (relu) return x > 0.0f ? 1.0f : 0.0f;
    float u = kGeluC * (x + kGeluA * x * x * x);
    float t = std::tanh(u);
    return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * kGeluC * (1.0f + 3.0f * kGeluA * x * x);
}

// Causal multi-head attention forward (cpu_model.cpp:148-180) for one batch of
// B sequences of S tokens.  q, k, v, o are [B*S, ld] with head h at column h*dh.
// P (softmax probabilities) is kept for the backward: [B, H, S, S].
void attn_fwd(float* o, float* P, const float* q, const float* k, const float* v, int ldq, int ldo, int B, int S,
              int H, int dh) {
    const float scale = 1.0f / std::sqrt((float)dh);
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < H; ++h) {
            float* Pb = P + ((size_t)(b * H + h)) * S * S;
            for (int i = 0; i < S; ++i) {
                const float* qi = q + (size_t)(b * S + i) * ldq + h * dh;
                float* pr = Pb + (size_t)i * S;
                float mx = -1e30f;
                for (int j = 0; j < S; ++j) {
                    float s;
                    if (j > i) s = -1e9f;
                    else {
                        const float* kj = k + (size_t)(b * S + j) * ldq + h * dh;
                        float acc = 0.0f;
                        for (int d = 0; d < dh; ++d) acc += qi[d] * kj[d];
                        s = acc * scale;
                    }
                    pr[j] = s;
                    mx = std::max(mx, s);
                }
                float sum = 0.0f;
                for (int j = 0; j < S; ++j) { pr[j] = std::exp(pr[j] - mx); sum += pr[j]; }
                for (int j = 0; j < S; ++j) pr[j] /= sum;
                float* oi = o + (size_t)(b * S + i) * ldo + h * dh;
                for (int d = 0; d < dh; ++d) oi[d] = 0.0f;
                for (int j = 0; j <= i; ++j) {
                    const float* vj = v + (size_t)(b * S + j) * ldq + h * dh;
                    for (int d = 0; d < dh; ++d) oi[d] += pr[j] * vj[d];
                }
            }
        }
}

// Backward of attn_fwd: dV = P^T dO, dP = dO V^T, dS = P (dP - rowsum(dP P)),
// dQ = dS K scale, dK = dS^T Q scale.  dq/dk/dv written (same layout as q/k/v).
void attn_bwd(float* dq, float* dk, float* dv, const float* dout, const float* P, const float* q, const float* k,
              const float* v, int ldq, int ldo, int B, int S, int H, int dh) {
    const float scale = 1.0f / std::sqrt((float)dh);
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < H; ++h) {
            const float* Pb = P + ((size_t)(b * H + h)) * S * S;
            std::vector<float> dS((size_t)S * S, 0.0f);
            for (int i = 0; i < S; ++i) {
                const float* doi = dout + (size_t)(b * S + i) * ldo + h * dh;
                const float* pr = Pb + (size_t)i * S;
                float dot = 0.0f;
                for (int j = 0; j <= i; ++j) {
                    const float* vj = v + (size_t)(b * S + j) * ldq + h * dh;
                    float dp = 0.0f;
                    for (int d = 0; d < dh; ++d) dp += doi[d] * vj[d];
                    dS[(size_t)i * S + j] = dp;
                    dot += dp * pr[j];
                }
                for (int j = 0; j <= i; ++j) dS[(size_t)i * S + j] = pr[j] * (dS[(size_t)i * S + j] - dot);
            }
            for (int i = 0; i < S; ++i) {
                float* dqi = dq + (size_t)(b * S + i) * ldq + h * dh;
                for (int d = 0; d < dh; ++d) dqi[d] = 0.0f;
                for (int j = 0; j <= i; ++j) {
                    const float* kj = k + (size_t)(b * S + j) * ldq + h * dh;
                    const float s = dS[(size_t)i * S + j] * scale;
                    for (int d = 0; d < dh; ++d) dqi[d] += s * kj[d];
                }
            }
            for (int j = 0; j < S; ++j) {
                float* dkj = dk + (size_t)(b * S + j) * ldq + h * dh;
                float* dvj = dv + (size_t)(b * S + j) * ldq + h * dh;
                for (int d = 0; d < dh; ++d) { dkj[d] = 0.0f; dvj[d] = 0.0f; }
                for (int i = j; i < S; ++i) {
                    const float* qi = q + (size_t)(b * S + i) * ldq + h * dh;
                    const float* doi = dout + (size_t)(b * S + i) * ldo + h * dh;
                    const float s = dS[(size_t)i * S + j] * scale;
                    const float p = Pb[(size_t)i * S + j];
                    for (int d = 0; d < dh; ++d) { dkj[d] += s * qi[d]; dvj[d] += p * doi[d]; }
                }
            }
        }
}

struct LoraView {   // rank-r adapters on the Q and V projections (cpu_lora.h:16-47 layout)
    int r;
    float scaling;
    const float* A[2];   // [D, r] per layer, stacked: A[l*D*r]
    const float* Bm[2];  // [r, D]
    float* dA[2];
    float* dB[2];
};

}  // namespace

extern "C" {

// ----------------------------- single ops ----------------------------------

void ora_gemm(int M, int N, int K, const float* A, int lda, int tA, const float* B, int ldb, int tB, float* C,
              int ldc, float beta) {
    gemm(M, N, K, A, lda, tA != 0, B, ldb, tB != 0, C, ldc, beta);
}

void ora_ln_fwd(float* y, float* mean, float* rstd, const float* x, const float* g, const float* b, int N, int D,
                float eps) {
    ln_fwd(y, mean, rstd, x, g, b, N, D, eps);
}

// dx = LN backward (+ dres when dres != nullptr); dg, db accumulate.
// ref_formula != 0 selects the reference's dx expression (see ln_bwd).
void ora_ln_bwd(float* dx, float* dg, float* db, const float* dy, const float* dres, const float* x, const float* g,
                const float* mean, const float* rstd, int N, int D, int ref_formula) {
    if (dres) std::memcpy(dx, dres, sizeof(float) * (size_t)N * D);
    ln_bwd(dx, dres != nullptr, dg, db, dy, x, g, mean, rstd, N, D, ref_formula != 0);
}

// Row softmax backward, cpu_mat.h:190-200: dx = y (dy - <dy, y>).
void ora_softmax_bwd(float* dx, const float* dy, const float* y, int N, int C) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < N; ++i) {
        float dot = 0.0f;
        for (int j = 0; j < C; ++j) dot += dy[(size_t)i * C + j] * y[(size_t)i * C + j];
        for (int j = 0; j < C; ++j) dx[(size_t)i * C + j] = y[(size_t)i * C + j] * (dy[(size_t)i * C + j] - dot);
    }
}

// Causal attention-softmax backward over nmat stacked [T, T] matrices: row i
// only covers columns j <= i (the strict upper triangle of dx is set to 0).
void ora_causal_softmax_bwd(float* dx, const float* dy, const float* y, int nmat, int T) {
#pragma omp parallel for schedule(static)
    for (long r = 0; r < (long)nmat * T; ++r) {
        const int i = (int)(r % T);
        const float* yr = y + (size_t)r * T;
        const float* dyr = dy + (size_t)r * T;
        float* dxr = dx + (size_t)r * T;
        float dot = 0.0f;
        for (int j = 0; j <= i; ++j) dot += dyr[j] * yr[j];
        for (int j = 0; j < T; ++j) dxr[j] = j <= i ? yr[j] * (dyr[j] - dot) : 0.0f;
    }
}

// Cross-entropy forward, cpu_mat.h:203-217.  Returns the mean loss; per-row
// losses and log-sum-exp are written when the pointers are non-null.
float ora_ce_fwd(const float* logits, const int* tgt, int N, int V, float* row_loss, float* row_lse) {
    double total = 0.0;
#pragma omp parallel for reduction(+ : total) schedule(static)
    for (int i = 0; i < N; ++i) {
        const float* z = logits + (size_t)i * V;
        float mx = -1e30f;
        for (int j = 0; j < V; ++j) mx = std::max(mx, z[j]);
        float s = 0.0f;
        for (int j = 0; j < V; ++j) s += std::exp(z[j] - mx);
        float lp = z[tgt[i]] - mx - std::log(s + 1e-10f);
        if (row_loss) row_loss[i] = -lp;
        if (row_lse) row_lse[i] = mx + std::log(s);
        total += -lp;
    }
    return (float)(total / N);
}

// Cross-entropy backward, cpu_mat.h:220-236, with the upstream scale folded in:
// d = (softmax(z) - onehot(t)) / N * scale.
void ora_ce_bwd(float* dlogits, const float* logits, const int* tgt, int N, int V, float scale) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < N; ++i) {
        const float* z = logits + (size_t)i * V;
        float mx = -1e30f;
        for (int j = 0; j < V; ++j) mx = std::max(mx, z[j]);
        float s = 0.0f;
        for (int j = 0; j < V; ++j) s += std::exp(z[j] - mx);
        for (int j = 0; j < V; ++j) {
            float p = std::exp(z[j] - mx) / s;
            dlogits[(size_t)i * V + j] = (p - (j == tgt[i] ? 1.0f : 0.0f)) / N * scale;
        }
    }
}

// Embedding backward, cpu_mat.h:265-277: dW[idx[t]] += dout[t] (accumulates).
void ora_embed_bwd(float* dW, const float* dout, const int* idx, int T, int D) {
    for (int t = 0; t < T; ++t)
        for (int d = 0; d < D; ++d) dW[(size_t)idx[t] * D + d] += dout[(size_t)t * D + d];
}

// AdamW with L2-coupled decay and pow bias correction, cpu_mat.h:280-292.
void ora_adamw(float* p, const float* g, float* m, float* v, long n, float lr, float b1, float b2, float eps,
               float wd, int t) {
    const float c1 = 1.0f - std::pow(b1, (float)t), c2 = 1.0f - std::pow(b2, (float)t);
#pragma omp parallel for schedule(static)
    for (long i = 0; i < n; ++i) {
        float gi = g[i] + wd * p[i];
        m[i] = b1 * m[i] + (1.0f - b1) * gi;
        v[i] = b2 * v[i] + (1.0f - b2) * gi * gi;
        float mh = m[i] / c1, vh = v[i] / c2;
        p[i] -= lr * mh / (std::sqrt(vh) + eps);
    }
}

// Per-tensor L2 clip, cpu_mat.h:295-306.  Returns the pre-clip norm.
float ora_clip(float* g, long n, float max_norm) {
    double s = 0.0;
    for (long i = 0; i < n; ++i) s += (double)g[i] * g[i];
    float norm = (float)std::sqrt(s);
    if (norm > max_norm) {
        float sc = max_norm / norm;
        for (long i = 0; i < n; ++i) g[i] *= sc;
    }
    return norm;
}

// Dynamic loss scaler, cuda_kernels.cu:102-116 (backoff 0.5, growth 2 every
// `interval` clean steps, clamp [1, 65536]).  state = {scale, unskipped(int as float)}.
// Returns 1 when the step must be skipped.
struct ora_scaler { float scale; int unskipped; int interval; };
int ora_scaler_update(ora_scaler* s, int overflow) {
    if (overflow) {
        s->unskipped = 0;
        s->scale *= 0.5f;
        if (s->scale < 1.0f) s->scale = 1.0f;
        return 1;
    }
    s->unskipped++;
    if (s->unskipped >= s->interval) {
        s->scale *= 2.0f;
        if (s->scale > 65536.0f) s->scale = 65536.0f;
        s->unskipped = 0;
    }
    return 0;
}

// Fused mixed-precision tail over the whole arena: overflow check on the scaled
// gradients, unscale, optional per-tensor clip, AdamW, scaler update, gradient
// zeroing.  seg_off/seg_len give the tensors (for clipping).  Returns 1 on skip.
int ora_adam_tail(float* p, float* g, float* m, float* v, long n, const long* seg_off, const long* seg_len,
                  int nseg, float lr, float b1, float b2, float eps, float wd, int t, ora_scaler* sc,
                  float max_norm) {
    int overflow = 0;
    for (long i = 0; i < n; ++i)
        if (!std::isfinite(g[i])) { overflow = 1; break; }
    if (!overflow) {
        const float inv = 1.0f / sc->scale;
        for (long i = 0; i < n; ++i) g[i] *= inv;
        if (max_norm > 0.0f)
            for (int s = 0; s < nseg; ++s) ora_clip(g + seg_off[s], seg_len[s], max_norm);
        ora_adamw(p, g, m, v, n, lr, b1, b2, eps, wd, t);
    }
    int skip = ora_scaler_update(sc, overflow);
    std::memset(g, 0, sizeof(float) * (size_t)n);
    return skip;
}

void ora_act_fwd(float* y, const float* x, long n, int relu) {
    for (long i = 0; i < n; ++i) y[i] = act_fwd(x[i], relu);
}
void ora_act_grad(float* y, const float* x, long n, int relu) {
    for (long i = 0; i < n; ++i) y[i] = act_grad(x[i], relu);
}

void ora_attn_fwd(float* o, float* P, const float* q, const float* k, const float* v, int ldq, int ldo, int B,
                  int S, int H, int dh) {
    attn_fwd(o, P, q, k, v, ldq, ldo, B, S, H, dh);
}
void ora_attn_bwd(float* dq, float* dk, float* dv, const float* dout, const float* P, const float* q,
                  const float* k, const float* v, int ldq, int ldo, int B, int S, int H, int dh) {
    attn_bwd(dq, dk, dv, dout, P, q, k, v, ldq, ldo, B, S, H, dh);
}

// ----------------------------- full model ----------------------------------
//
// Loss and gradients of the decoder for B sequences of S tokens.
//   params: flat FP32 arena (rbk_layout.h order).
//   grads : flat arena, overwritten (zeroed then filled) unless lora != null,
//           in which case base gradients are not produced at all.
//   grad_scale: upstream multiplier on dlogits (the dynamic loss scale, or the
//           reference's 1/(BS*GA) argument, model.cu:349-350).
//   act_relu: 1 = ReLU FFN (reference behaviour), 0 = GELU (this build).
//   logits_out (optional): [B*S, V] FP32 logits.
// Returns the mean cross-entropy.
static float model_loss_grad(const rbk_config* c, const float* params, float* grads, const int* tok,
                             const int* tgt, int B, int S, float grad_scale, int act_relu, float* logits_out,
                             LoraView* lora) {
    const int N = B * S, D = c->D, F = c->FF, V = c->V, H = c->H, L = c->L, dh = D / H;
    std::vector<rbk_tensor> tab(rbk_num_tensors(c));
    const int64_t nparams = rbk_param_table(c, tab.data());
    auto P = [&](int idx) { return params + tab[idx].offset; };
    auto G = [&](int idx) { return grads + tab[idx].offset; };
    const bool base_grads = (lora == nullptr) && grads;
    if (base_grads) std::memset(grads, 0, sizeof(float) * (size_t)nparams);

    struct LA {
        std::vector<float> x, h1, mu1, rs1, qkv, o, Pm, x1, h2, mu2, rs2, pre, a, xa;  // xa: h1 A (lora)
    };
    std::vector<LA> la(L);
    std::vector<float> x0((size_t)N * D);
    for (int n = 0; n < N; ++n)
        for (int d = 0; d < D; ++d)
            x0[(size_t)n * D + d] = P(RBK_TOK_EMB)[(size_t)tok[n] * D + d] + P(RBK_POS_EMB)[(size_t)(n % S) * D + d];

    std::vector<float> xcur = x0;
    for (int l = 0; l < L; ++l) {
        auto& A = la[l];
        auto W = [&](int j) { return P(rbk_layer_tensor(l, j)); };
        A.x = xcur;
        A.h1.resize((size_t)N * D); A.mu1.resize(N); A.rs1.resize(N);
        ln_fwd(A.h1.data(), A.mu1.data(), A.rs1.data(), A.x.data(), W(RBK_LN1_W), W(RBK_LN1_B), N, D, 1e-5f);
        A.qkv.resize((size_t)N * 3 * D);
        linear(A.qkv.data(), A.h1.data(), W(RBK_WQ), W(RBK_BQ), N, D, 3 * D);   // wq|wk|wv adjacent
        if (lora) {
            const int r = lora->r;
            A.xa.resize((size_t)N * 2 * r);
            for (int t = 0; t < 2; ++t) {   // t=0 -> Q (column block 0), t=1 -> V (column block 2)
                const float* Al = lora->A[t] + (size_t)l * D * r;
                const float* Bl = lora->Bm[t] + (size_t)l * r * D;
                std::vector<float> xa((size_t)N * r), add((size_t)N * D);
                gemm(N, r, D, A.h1.data(), D, false, Al, r, false, xa.data(), r, 0.0f);
                gemm(N, D, r, xa.data(), r, false, Bl, D, false, add.data(), D, 0.0f);
                const int col = t == 0 ? 0 : 2 * D;
                for (int n = 0; n < N; ++n) {
                    for (int d = 0; d < D; ++d) A.qkv[(size_t)n * 3 * D + col + d] += lora->scaling * add[(size_t)n * D + d];
                    for (int j = 0; j < r; ++j) A.xa[(size_t)n * 2 * r + t * r + j] = xa[(size_t)n * r + j];
                }
            }
        }
        A.o.resize((size_t)N * D);
        A.Pm.resize((size_t)B * H * S * S);
        attn_fwd(A.o.data(), A.Pm.data(), A.qkv.data(), A.qkv.data() + D, A.qkv.data() + 2 * D, 3 * D, D, B, S, H,
                 dh);
        A.x1.resize((size_t)N * D);
        linear(A.x1.data(), A.o.data(), W(RBK_WO), W(RBK_BO), N, D, D);
        for (size_t i = 0; i < A.x1.size(); ++i) A.x1[i] += A.x[i];
        A.h2.resize((size_t)N * D); A.mu2.resize(N); A.rs2.resize(N);
        ln_fwd(A.h2.data(), A.mu2.data(), A.rs2.data(), A.x1.data(), W(RBK_LN2_W), W(RBK_LN2_B), N, D, 1e-5f);
        A.pre.resize((size_t)N * F); A.a.resize((size_t)N * F);
        linear(A.pre.data(), A.h2.data(), W(RBK_W1), W(RBK_B1), N, D, F);
        for (size_t i = 0; i < A.pre.size(); ++i) A.a[i] = act_fwd(A.pre[i], act_relu);
        std::vector<float> y((size_t)N * D);
        linear(y.data(), A.a.data(), W(RBK_W2), W(RBK_B2), N, F, D);
        for (size_t i = 0; i < y.size(); ++i) xcur[i] = A.x1[i] + y[i];
    }
    const int iLNW = rbk_tail_tensor(c, RBK_LN_F_W), iLNB = rbk_tail_tensor(c, RBK_LN_F_B);
    const int iLMW = rbk_tail_tensor(c, RBK_LM_W), iLMB = rbk_tail_tensor(c, RBK_LM_B);
    std::vector<float> hf((size_t)N * D), muf(N), rsf(N), logits((size_t)N * V);
    ln_fwd(hf.data(), muf.data(), rsf.data(), xcur.data(), P(iLNW), P(iLNB), N, D, 1e-5f);
    linear(logits.data(), hf.data(), P(iLMW), P(iLMB), N, D, V);
    if (logits_out) std::memcpy(logits_out, logits.data(), sizeof(float) * logits.size());
    const float loss = ora_ce_fwd(logits.data(), tgt, N, V, nullptr, nullptr);
    if (!grads && !lora) return loss;

    // ------------------------------ backward ------------------------------
    std::vector<float>& dlog = logits;   // reuse storage
    {
        std::vector<float> tmp((size_t)N * V);
        ora_ce_bwd(tmp.data(), logits.data(), tgt, N, V, grad_scale);
        dlog.swap(tmp);
    }
    std::vector<float> dhf((size_t)N * D);
    linear_bwd(dhf.data(), false, base_grads ? G(iLMW) : nullptr, base_grads ? G(iLMB) : nullptr, dlog.data(),
               hf.data(), P(iLMW), N, D, V);
    std::vector<float> dx((size_t)N * D), scratch_g(2 * (size_t)D);
    float* gLNW = base_grads ? G(iLNW) : scratch_g.data();
    float* gLNB = base_grads ? G(iLNB) : scratch_g.data() + D;
    ln_bwd(dx.data(), false, gLNW, gLNB, dhf.data(), xcur.data(), P(iLNW), muf.data(), rsf.data(), N, D);

    std::vector<float> scr_dg(2 * (size_t)D);
    for (int l = L - 1; l >= 0; --l) {
        auto& A = la[l];
        auto W = [&](int j) { return P(rbk_layer_tensor(l, j)); };
        auto GW = [&](int j) { return base_grads ? G(rbk_layer_tensor(l, j)) : nullptr; };
        // FFN
        std::vector<float> da((size_t)N * F), dh2((size_t)N * D);
        linear_bwd(da.data(), false, GW(RBK_W2), GW(RBK_B2), dx.data(), A.a.data(), W(RBK_W2), N, F, D);
        for (size_t i = 0; i < da.size(); ++i) da[i] *= act_grad(A.pre[i], act_relu);
        linear_bwd(dh2.data(), false, GW(RBK_W1), GW(RBK_B1), da.data(), A.h2.data(), W(RBK_W1), N, D, F);
        std::vector<float> dx1 = dx;   // residual branch
        ln_bwd(dx1.data(), true, GW(RBK_LN2_W) ? GW(RBK_LN2_W) : scr_dg.data(),
               GW(RBK_LN2_B) ? GW(RBK_LN2_B) : scr_dg.data() + D, dh2.data(), A.x1.data(), W(RBK_LN2_W),
               A.mu2.data(), A.rs2.data(), N, D);
        // attention output projection
        std::vector<float> dO((size_t)N * D);
        linear_bwd(dO.data(), false, GW(RBK_WO), GW(RBK_BO), dx1.data(), A.o.data(), W(RBK_WO), N, D, D);
        // attention core
        std::vector<float> dqkv((size_t)N * 3 * D);
        attn_bwd(dqkv.data(), dqkv.data() + D, dqkv.data() + 2 * D, dO.data(), A.Pm.data(), A.qkv.data(),
                 A.qkv.data() + D, A.qkv.data() + 2 * D, 3 * D, D, B, S, H, dh);
        // QKV projection (one [3D, D] GEMM)
        std::vector<float> dh1((size_t)N * D);
        linear_bwd(dh1.data(), false, GW(RBK_WQ), GW(RBK_BQ), dqkv.data(), A.h1.data(), W(RBK_WQ), N, D, 3 * D);
        if (lora) {
            const int r = lora->r;
            for (int t = 0; t < 2; ++t) {
                const float* Al = lora->A[t] + (size_t)l * D * r;
                const float* Bl = lora->Bm[t] + (size_t)l * r * D;
                float* dAl = lora->dA[t] + (size_t)l * D * r;
                float* dBl = lora->dB[t] + (size_t)l * r * D;
                const int col = t == 0 ? 0 : 2 * D;
                std::vector<float> dy((size_t)N * D), xa((size_t)N * r), dyB((size_t)N * r);
                for (int n = 0; n < N; ++n) {
                    for (int d = 0; d < D; ++d) dy[(size_t)n * D + d] = lora->scaling * dqkv[(size_t)n * 3 * D + col + d];
                    for (int j = 0; j < r; ++j) xa[(size_t)n * r + j] = A.xa[(size_t)n * 2 * r + t * r + j];
                }
                // dB += (xA)^T (s dy) ; dyB = (s dy) B^T ; dA += x^T dyB ; dh1 += dyB A^T
                gemm(r, D, N, xa.data(), r, true, dy.data(), D, false, dBl, D, 1.0f);
                gemm(N, r, D, dy.data(), D, false, Bl, D, true, dyB.data(), r, 0.0f);
                gemm(D, r, N, A.h1.data(), D, true, dyB.data(), r, false, dAl, r, 1.0f);
                gemm(N, D, r, dyB.data(), r, false, Al, r, true, dh1.data(), D, 1.0f);
            }
        }
        std::vector<float> dxn = dx1;
        ln_bwd(dxn.data(), true, GW(RBK_LN1_W) ? GW(RBK_LN1_W) : scr_dg.data(),
               GW(RBK_LN1_B) ? GW(RBK_LN1_B) : scr_dg.data() + D, dh1.data(), A.x.data(), W(RBK_LN1_W),
               A.mu1.data(), A.rs1.data(), N, D);
        dx.swap(dxn);
    }
    if (base_grads) {
        ora_embed_bwd(G(RBK_TOK_EMB), dx.data(), tok, N, D);
        float* gp = G(RBK_POS_EMB);
        for (int n = 0; n < N; ++n)
            for (int d = 0; d < D; ++d) gp[(size_t)(n % S) * D + d] += dx[(size_t)n * D + d];
    }
    return loss;
}

// cfg6 = {V, T, D, H, L, FF}
float ora_model_loss_grad(const int* cfg6, const float* params, float* grads, const int* tok, const int* tgt,
                          int B, int S, float grad_scale, int act_relu, float* logits_out) {
    rbk_config c{cfg6[0], cfg6[1], cfg6[2], cfg6[3], cfg6[4], cfg6[5]};
    return model_loss_grad(&c, params, grads, tok, tgt, B, S, grad_scale, act_relu, logits_out, nullptr);
}

// LoRA fine-tune backward on frozen base weights: gradients only to the Q and
// V adapters (A [D, r], B [r, D] per layer, stacked over layers), scaling alpha/r.
float ora_model_lora_grad(const int* cfg6, const float* params, const float* Aq, const float* Bq, const float* Av,
                          const float* Bv, float* dAq, float* dBq, float* dAv, float* dBv, int r, float alpha,
                          const int* tok, const int* tgt, int B, int S, float grad_scale) {
    rbk_config c{cfg6[0], cfg6[1], cfg6[2], cfg6[3], cfg6[4], cfg6[5]};
    LoraView lv;
    lv.r = r; lv.scaling = alpha / r;
    lv.A[0] = Aq; lv.A[1] = Av; lv.Bm[0] = Bq; lv.Bm[1] = Bv;
    lv.dA[0] = dAq; lv.dA[1] = dAv; lv.dB[0] = dBq; lv.dB[1] = dBv;
    const size_t na = (size_t)c.L * c.D * r;
    std::memset(dAq, 0, na * 4); std::memset(dAv, 0, na * 4);
    std::memset(dBq, 0, na * 4); std::memset(dBv, 0, na * 4);
    return model_loss_grad(&c, params, nullptr, tok, tgt, B, S, grad_scale, 0, nullptr, &lv);
}

long ora_num_params(const int* cfg6) {
    rbk_config c{cfg6[0], cfg6[1], cfg6[2], cfg6[3], cfg6[4], cfg6[5]};
    return (long)rbk_num_params(&c);
}

int ora_param_table(const int* cfg6, long* off_rows_cols) {
    rbk_config c{cfg6[0], cfg6[1], cfg6[2], cfg6[3], cfg6[4], cfg6[5]};
    std::vector<rbk_tensor> t(rbk_num_tensors(&c));
    rbk_param_table(&c, t.data());
    for (size_t i = 0; i < t.size(); ++i) {
        off_rows_cols[3 * i] = t[i].offset;
        off_rows_cols[3 * i + 1] = t[i].rows;
        off_rows_cols[3 * i + 2] = t[i].cols;
    }
    return (int)t.size();
}

int ora_num_threads(void) { return omp_get_max_threads(); }
// Thread count for the following calls (torchrun exports OMP_NUM_THREADS=1 to every rank).
void ora_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}

}  // extern "C"
