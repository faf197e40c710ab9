// lora.cu — kernel-level LoRA adapter entry points, for callers that keep their own
// orchestration (the model-level path runs the same GEMMs inside rbk_model_forward /
// rbk_model_backward).  One adapter on one projection, W' = W + scaling * A B with
// A [in, r] and B [r, out] row-major FP16 (the per-target step of lora_forward_all /
// lora_backward_all, src/lora.h:223-229, and the math of src/cpu_lora.h):
//
//   forward:  xa = x A;  y += scaling * xa B
//   backward: dB += scaling * xa^T dy;  dyb = scaling * dy B^T;  dA += x^T dyb;  dx += dyb A^T
//
// Every product is one rbk_gemm (tcgen05 tiles, FP32 accumulation); the additions into y and
// dx ride on the FP16 epilogue's residual input, the gradient accumulations on the FP32
// accumulate epilogue.  lora_optimizer_step (src/lora.h:230) is the fused AdamW tail over the
// adapter arena.
#include "common.cuh"

namespace rbk {
namespace {

// role: the profiler's GEMM category (0 forward, 1 dgrad, 2 wgrad)
int gemm(rbk_ctx* ctx, cudaStream_t st, int role, int M, int N, int K, const void* A, int lda, int am, const void* B,
         int ldb, int bm, void* C, int ldc, int epi, const void* aux, int ld_aux, float alpha) {
    rbk_gemm_desc d = {};
    d.M = M; d.N = N; d.K = K;
    d.A = A; d.lda = lda; d.a_major = am;
    d.B = B; d.ldb = ldb; d.b_major = bm;
    d.C = C; d.ldc = ldc;
    d.epilogue = epi;
    d.aux = aux; d.ld_aux = ld_aux;
    d.alpha = alpha;
    const int saved = ctx->gemm_role;
    ctx->gemm_role = role;
    const int r = rbk_gemm(ctx, &d, st);
    ctx->gemm_role = saved;
    return r;
}

}  // namespace
}  // namespace rbk

using namespace rbk;

extern "C" {

int rbk_lora_fwd(rbk_ctx* ctx, void* y, int ldy, void* xa, const void* x, int ldx, const void* A, const void* B,
                 int N, int in, int r, int out, float scaling, void* stream) {
    RBK_REQUIRE(ctx && y && xa && x && A && B, "rbk_lora_fwd: null pointer");
    RBK_REQUIRE(N > 0 && in > 0 && out > 0 && r > 0 && r % 8 == 0 && in % 8 == 0 && out % 8 == 0,
                "rbk_lora_fwd: need N, in, out, r > 0 and in, out, r multiples of 8");
    RBK_REQUIRE(ldx >= in && ldy >= out && ldx % 8 == 0 && ldy % 8 == 0, "rbk_lora_fwd: bad row strides");
    cudaStream_t st = as_stream(stream);
    // xa[N, r] = x A   (A [in, r]: B operand (n = j, k = d) = A[d r + j], MN-major)
    RBK_TRY(gemm(ctx, st, 0, N, r, in, x, ldx, 0, A, r, 1, xa, r, RBK_EPI_STORE_F16, nullptr, 0, 1.0f));
    // y += scaling * xa B   (B [r, out]: (n = o, k = j) = B[j out + o], MN-major), in place
    return gemm(ctx, st, 0, N, out, r, xa, r, 0, B, out, 1, y, ldy, RBK_EPI_STORE_F16, y, ldy, scaling);
}

int rbk_lora_bwd(rbk_ctx* ctx, float* dA, float* dB, void* dx, int lddx, void* dyb, const void* dy, int lddy,
                 const void* x, int ldx, const void* xa, const void* A, const void* B, int N, int in, int r, int out,
                 float scaling, void* stream) {
    RBK_REQUIRE(ctx && dA && dB && dyb && dy && x && xa && A && B, "rbk_lora_bwd: null pointer");
    RBK_REQUIRE(N > 0 && in > 0 && out > 0 && r > 0 && r % 8 == 0 && in % 8 == 0 && out % 8 == 0,
                "rbk_lora_bwd: need N, in, out, r > 0 and in, out, r multiples of 8");
    RBK_REQUIRE(ldx >= in && lddy >= out && ldx % 8 == 0 && lddy % 8 == 0 && (!dx || (lddx >= in && lddx % 8 == 0)),
                "rbk_lora_bwd: bad row strides");
    cudaStream_t st = as_stream(stream);
    // dB[r, out] += scaling * xa^T dy
    RBK_TRY(gemm(ctx, st, 2, r, out, N, xa, r, 1, dy, lddy, 1, dB, out, RBK_EPI_ACC_F32, nullptr, 0, scaling));
    // dyb[N, r] = scaling * dy B^T   ((n = j, k = o) = B[j out + o], K-major)
    RBK_TRY(gemm(ctx, st, 1, N, r, out, dy, lddy, 0, B, out, 0, dyb, r, RBK_EPI_STORE_F16, nullptr, 0, scaling));
    // dA[in, r] += x^T dyb
    RBK_TRY(gemm(ctx, st, 2, in, r, N, x, ldx, 1, dyb, r, 1, dA, r, RBK_EPI_ACC_F32, nullptr, 0, 1.0f));
    // dx[N, in] += dyb A^T   ((n = d, k = j) = A[d r + j], K-major), in place
    if (dx) RBK_TRY(gemm(ctx, st, 1, N, in, r, dyb, r, 0, A, r, 0, dx, lddx, RBK_EPI_STORE_F16, dx, lddx, 1.0f));
    return RBK_OK;
}

int rbk_lora_adam(rbk_ctx* ctx, const rbk_tail_args* args, void* stream) {
    RBK_REQUIRE(args, "rbk_lora_adam: null arguments");
    return rbk_adam_tail(ctx, args, stream);
}

}  // extern "C"
