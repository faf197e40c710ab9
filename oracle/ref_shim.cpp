// ref_shim.cpp — C entry points onto the reference's own CPU engine, compiled
// from the reference sources where they lie (see oracle/Makefile, target
// `ref`).  Output goes to oracle/_ref/libref.so, which is git-ignored.
//
// TEST INFRASTRUCTURE ONLY: used to pin the oracle restatement (oracle.cpp)
// and to generate the golden fixtures under tests/golden/.  The reference
// engine only builds without -fopenmp (src/cpu_mat.h:134 is rejected by g++ 13
// under OpenMP), so everything here runs serially.
//
// Wrapped reference functions:
//   cpuops::layer_norm / layer_norm_backward   src/cpu_mat.h:98-153
//   cpuops::softmax / softmax_backward         src/cpu_mat.h:172-200
//   cpuops::cross_entropy / _backward          src/cpu_mat.h:203-236
//   cpuops::embedding_backward                 src/cpu_mat.h:265-277
//   cpuops::adamw_step                         src/cpu_mat.h:280-292
//   cpuops::clip_gradients                     src/cpu_mat.h:295-306
//   cpuops::matmul / matmul_tB / matmul_tA     src/cpu_mat.h:47-95
//   CPUTransformer::forward                    src/cpu_model.cpp:115-222
#include <chrono>
#include <cstring>
#include <vector>

#include "cpu_model.h"

namespace {
Mat mk(const float* p, int r, int c) {
    Mat m(r, c);
    std::memcpy(m.data.data(), p, sizeof(float) * (size_t)r * c);
    return m;
}
void out(float* dst, const Mat& m) { std::memcpy(dst, m.data.data(), sizeof(float) * m.data.size()); }
double secs(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}
}  // namespace

extern "C" {

void ref_layer_norm(float* y, float* mean, float* rstd, const float* x, const float* g, const float* b, int N,
                    int D) {
    Mat Y, M, R;
    cpuops::layer_norm(Y, M, R, mk(x, N, D), mk(g, 1, D), mk(b, 1, D));
    out(y, Y); out(mean, M); out(rstd, R);
}

void ref_layer_norm_backward(float* dx, float* dg, float* db, const float* dy, const float* x, const float* g,
                             const float* mean, const float* rstd, int N, int D) {
    Mat DX, DG, DB;
    cpuops::layer_norm_backward(DX, DG, DB, mk(dy, N, D), mk(x, N, D), mk(g, 1, D), mk(mean, N, 1),
                                mk(rstd, N, 1));
    out(dx, DX); out(dg, DG); out(db, DB);
}

void ref_softmax(float* y, const float* x, int N, int C) {
    Mat Y;
    cpuops::softmax(Y, mk(x, N, C));
    out(y, Y);
}

void ref_softmax_backward(float* dx, const float* dy, const float* y, int N, int C) {
    Mat DX;
    cpuops::softmax_backward(DX, mk(dy, N, C), mk(y, N, C));
    out(dx, DX);
}

float ref_cross_entropy(const float* logits, const int* tgt, int N, int V) {
    std::vector<int> t(tgt, tgt + N);
    return cpuops::cross_entropy(mk(logits, N, V), t);
}

void ref_cross_entropy_backward(float* dlogits, const float* logits, const int* tgt, int N, int V) {
    std::vector<int> t(tgt, tgt + N);
    Mat D;
    cpuops::cross_entropy_backward(D, mk(logits, N, V), t);
    out(dlogits, D);
}

void ref_embedding_backward(float* dW, const float* dout, const int* idx, int T, int D, int V) {
    std::vector<int> t(idx, idx + T);
    Mat DW;
    cpuops::embedding_backward(DW, mk(dout, T, D), t, V);
    out(dW, DW);
}

void ref_adamw_step(float* p, const float* g, float* m, float* v, int n, float lr, float b1, float b2, float eps,
                    float wd, int t) {
    Mat P = mk(p, 1, n), M = mk(m, 1, n), Vv = mk(v, 1, n);
    cpuops::adamw_step(P, mk(g, 1, n), M, Vv, lr, b1, b2, eps, wd, t);
    out(p, P); out(m, M); out(v, Vv);
}

float ref_clip_gradients(float* g, int n, float max_norm) {
    Mat G = mk(g, 1, n);
    float norm = cpuops::clip_gradients(G, max_norm);
    out(g, G);
    return norm;
}

// C = A B (M,K)x(K,N); C += A B^T; C += A^T B — the three reference variants.
void ref_matmul(float* C, const float* A, const float* B, int M, int K, int N) {
    Mat c(M, N);
    cpuops::matmul(c, mk(A, M, K), mk(B, K, N));
    out(C, c);
}
void ref_matmul_tB(float* C, const float* A, const float* B, int M, int K, int N) {
    Mat c(M, N);
    cpuops::matmul_tB(c, mk(A, M, K), mk(B, N, K));
    out(C, c);
}
void ref_matmul_tA(float* C, const float* A, const float* B, int M, int K, int N) {
    Mat c(M, N);
    cpuops::matmul_tA(c, mk(A, K, M), mk(B, K, N));
    out(C, c);
}

// Loss of CPUTransformer::forward on one sequence.  Weights are given in the
// reference CPU engine's own [in, out] convention (cpu_model.cpp:135-137,
// 183, 197-206) and its LM head multiplies by lm_w as [in, out]
// (cpu_model.cpp:214), which is only shape-correct when V == D; callers must
// use V == D.  FFN activation is ReLU (cpu_model.cpp:198-200).
// Per layer l, `layer` holds 16 blocks in this order (each row-major):
//   ln1_w[D] ln1_b[D] wq[D,D] bq[D] wk[D,D] bk[D] wv[D,D] bv[D] wo[D,D] bo[D]
//   ln2_w[D] ln2_b[D] w1[D,FF] b1[FF] w2[FF,D] b2[D]
float ref_cpu_forward(int V, int T, int D, int H, int L, int FF, const float* tok_emb, const float* pos_emb,
                      const float* layers, const float* ln_f_w, const float* ln_f_b, const float* lm_w,
                      const float* lm_b, const int* tokens, const int* targets, int S) {
    CPUConfig cfg;
    cfg.init(V, T, D, H, L, FF);
    CPUTransformer m;
    m.init(cfg);
    m.allocate_activations(S);
    m.w.token_emb = mk(tok_emb, V, D);
    m.w.pos_emb = mk(pos_emb, T, D);
    const float* p = layers;
    auto take = [&](Mat& dst, int r, int c) { dst = mk(p, r, c); p += (size_t)r * c; };
    for (int l = 0; l < L; ++l) {
        auto& ly = m.w.layers[l];
        take(ly.ln1_w, 1, D); take(ly.ln1_b, 1, D);
        take(ly.wq, D, D); take(ly.bq, 1, D);
        take(ly.wk, D, D); take(ly.bk, 1, D);
        take(ly.wv, D, D); take(ly.bv, 1, D);
        take(ly.wo, D, D); take(ly.bo, 1, D);
        take(ly.ln2_w, 1, D); take(ly.ln2_b, 1, D);
        take(ly.w1, D, FF); take(ly.b1, 1, FF);
        take(ly.w2, FF, D); take(ly.b2, 1, D);
    }
    m.w.ln_f_w = mk(ln_f_w, 1, D);
    m.w.ln_f_b = mk(ln_f_b, 1, D);
    m.w.lm_w = mk(lm_w, V, D);
    m.w.lm_b = mk(lm_b, 1, V);
    std::vector<int> tk(tokens, tokens + S), tg(targets, targets + S);
    return m.forward(tk, &tg);
}

// ---- timed variants for the CPU baseline: inputs are copied into the engine's
// matrices first, then only the reference call itself is timed (seconds).
double ref_time_layer_norm_backward(const float* dy, const float* x, const float* g, const float* mean,
                                    const float* rstd, int N, int D) {
    Mat DY = mk(dy, N, D), X = mk(x, N, D), G = mk(g, 1, D), M = mk(mean, N, 1), R = mk(rstd, N, 1);
    Mat DX, DG, DB;
    const auto t0 = std::chrono::steady_clock::now();
    cpuops::layer_norm_backward(DX, DG, DB, DY, X, G, M, R);
    return secs(t0);
}

double ref_time_softmax_backward(const float* dy, const float* y, int N, int C) {
    Mat DY = mk(dy, N, C), Y = mk(y, N, C), DX;
    const auto t0 = std::chrono::steady_clock::now();
    cpuops::softmax_backward(DX, DY, Y);
    return secs(t0);
}

double ref_time_cross_entropy_backward(const float* logits, const int* tgt, int N, int V) {
    Mat Z = mk(logits, N, V), D;
    std::vector<int> t(tgt, tgt + N);
    const auto t0 = std::chrono::steady_clock::now();
    cpuops::cross_entropy_backward(D, Z, t);
    return secs(t0);
}

double ref_time_adamw_step(const float* p, const float* g, int n, float lr, float b1, float b2, float eps, float wd) {
    Mat P = mk(p, 1, n), G = mk(g, 1, n), M(1, n), Vv(1, n);
    const auto t0 = std::chrono::steady_clock::now();
    cpuops::adamw_step(P, G, M, Vv, lr, b1, b2, eps, wd, 1);
    return secs(t0);
}

// CPUTransformer::forward (with its loss) on one sequence of S tokens; the
// same weight blocks as ref_cpu_forward (V == D), only the forward timed.
double ref_time_cpu_forward(int V, int T, int D, int H, int L, int FF, const float* tok_emb, const float* pos_emb,
                            const float* layers, const float* ln_f_w, const float* ln_f_b, const float* lm_w,
                            const float* lm_b, const int* tokens, const int* targets, int S, float* loss) {
    CPUConfig cfg;
    cfg.init(V, T, D, H, L, FF);
    CPUTransformer m;
    m.init(cfg);
    m.allocate_activations(S);
    m.w.token_emb = mk(tok_emb, V, D);
    m.w.pos_emb = mk(pos_emb, T, D);
    const float* p = layers;
    auto take = [&](Mat& dst, int r, int c) { dst = mk(p, r, c); p += (size_t)r * c; };
    for (int l = 0; l < L; ++l) {
        auto& ly = m.w.layers[l];
        take(ly.ln1_w, 1, D); take(ly.ln1_b, 1, D);
        take(ly.wq, D, D); take(ly.bq, 1, D);
        take(ly.wk, D, D); take(ly.bk, 1, D);
        take(ly.wv, D, D); take(ly.bv, 1, D);
        take(ly.wo, D, D); take(ly.bo, 1, D);
        take(ly.ln2_w, 1, D); take(ly.ln2_b, 1, D);
        take(ly.w1, D, FF); take(ly.b1, 1, FF);
        take(ly.w2, FF, D); take(ly.b2, 1, D);
    }
    m.w.ln_f_w = mk(ln_f_w, 1, D);
    m.w.ln_f_b = mk(ln_f_b, 1, D);
    m.w.lm_w = mk(lm_w, V, D);
    m.w.lm_b = mk(lm_b, 1, V);
    std::vector<int> tk(tokens, tokens + S), tg(targets, targets + S);
    const auto t0 = std::chrono::steady_clock::now();
    *loss = m.forward(tk, &tg);
    return secs(t0);
}

}  // extern "C"
