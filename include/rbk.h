/*
 * rbk.h — C ABI of the B200 (sm_100a) backward-pass library for
 * rubidium-train (librbk.so).
 *
 * Conventions (all entry points):
 *   - extern "C", plain pointers and sizes; device pointers unless stated.
 *   - every call takes the CUDA stream it launches on (`stream`, a
 *     cudaStream_t passed as void*; NULL = legacy default stream) and returns
 *     an int status: RBK_OK (0) or a negative RBK_ERR_* code.  Nothing calls
 *     exit(); rbk_last_error() holds a message for the calling thread.
 *   - "half" tensors are IEEE binary16 (the reference's FP16 activations and
 *     weights, src/model.h:29-55); "float" tensors are FP32.
 *   - the caller owns every buffer.  Scratch comes from the rbk_ctx, which
 *     allocates it on first use at a given size (never during a call that
 *     already had enough) and keeps it until rbk_ctx_destroy.
 *   - one rbk_ctx per host thread / stream; calls on one ctx are not
 *     thread-safe.
 *
 * Each entry point names the reference interface it replaces; reference paths
 * are relative to the rubidium-train project.
 */
#ifndef RBK_H
#define RBK_H

#include <stddef.h>
#include <stdint.h>

#include "rbk_layout.h"

#ifdef __cplusplus
extern "C" {
#endif

#define RBK_OK 0
#define RBK_ERR_INVALID (-1)      /* bad argument (shape, alignment, null)   */
#define RBK_ERR_CUDA (-2)         /* a CUDA runtime / driver call failed      */
#define RBK_ERR_UNSUPPORTED (-3)  /* device is not sm_100 or shape unsupported */
#define RBK_ERR_TIMEOUT (-4)      /* a bounded device-side wait ran out       */
#define RBK_ERR_NCCL (-5)         /* an NCCL call failed                      */
#define RBK_ERR_NOMEM (-6)        /* device allocation failed                 */
#define RBK_ERR_IO (-7)           /* a file could not be opened, read or written */

typedef struct rbk_ctx rbk_ctx;

/* Message of the last failing call on this thread ("" when none). */
const char* rbk_last_error(void);
/* Library ABI version (bumped on incompatible changes). */
int rbk_version(void);

/* Context: device binding + scratch arena.  Fails with RBK_ERR_UNSUPPORTED on
 * anything but a compute capability 10.0 device.
 * Replaces init_handles()/MemPool (src/cuda_kernels.cuh:30,46-57). */
int rbk_ctx_create(rbk_ctx** out, int device);
int rbk_ctx_destroy(rbk_ctx* ctx);

/* Instrumentation (no counterpart in the reference, which times steps with
 * clock(), src/main.cpp:123,178):
 *   rbk_launch_count   kernels launched by librbk since load (all contexts);
 *   rbk_ctx_profile    enable (1) / disable (0) per-entry-point CUDA-event
 *                      timing on ctx and clear its records;
 *   rbk_ctx_profile_read  synchronise and sum per category (>= RBK_PROF_NCAT
 *                      slots): milliseconds, algorithmic work (GEMM and
 *                      attention FLOPs, bytes for the others) and launches.
 *                      Categories: 0 GEMM, 1 attention fwd, 2 attention bwd,
 *                      3 LN fwd, 4 LN bwd, 5 softmax-CE, 6 Adam tail,
 *                      7 embeddings, 8 other;
 *   rbk_ctx_device_error  read and clear the status word that bounded
 *                      device-side waits set (0 or RBK_ERR_TIMEOUT). */
#define RBK_PROF_NCAT 9
long long rbk_launch_count(void);
int rbk_ctx_profile(rbk_ctx* ctx, int enable);
int rbk_ctx_profile_read(rbk_ctx* ctx, double* ms, double* work, int* launches, int ncat);
/* The GEMM category split by role (3 slots each): 0 forward (and checkpoint
 * recompute), 1 data gradient (dgrad), 2 weight gradient (wgrad).  The model
 * tags every GEMM it issues; a direct rbk_gemm call counts as wgrad when its
 * epilogue accumulates / stores FP32, dgrad when B is MN-major, else forward. */
int rbk_ctx_profile_read_gemm(rbk_ctx* ctx, double* ms, double* flops, int* launches);
int rbk_ctx_device_error(rbk_ctx* ctx, int* status);
/* Bitwise-reproducible gradients (default off, or on for every new context when
 * RBK_DETERMINISTIC=1), so two runs on the same inputs give identical bits:
 *   - split-K weight-gradient GEMMs write one FP32 partial plane per split
 *     (ctx scratch), and a reduction launch adds them to C in split order,
 *     instead of FP32 atomics;
 *   - the tcgen05 attention backward adds each query block's dQ contributions
 *     in ascending key-block order (per-block counters);
 *   - the token-embedding gradient sums each token's rows in position order
 *     after a key sort (up to 32768 positions per call).
 * Measured cost on the GPT-2-small step: about 7% (the ordered dQ additions
 * and the split-K reductions).  No counterpart in the reference. */
int rbk_ctx_set_deterministic(rbk_ctx* ctx, int on);

/* Test only: arms the next rbk_adam_tail launch on this context (one launch; the
 * setting is cleared when it is used).  Its grid-barrier wait gives up after
 * limit_s seconds (1e-4 .. 2; the default is 2 s) and CTA `withheld_cta` does
 * not arrive at the barrier (-1: every CTA arrives; larger than the grid: the
 * last CTA), so that the bounded wait runs out on a healthy GPU.  The launch
 * then returns as for a timeout in production: the step is skipped like an
 * overflow step (masters and moments untouched, gradients zeroed, scale halved)
 * and rbk_scaler.status = RBK_ERR_TIMEOUT; the next launch runs normally.
 * It exercises the failure path of the bounded device waits without a GPU
 * fault.  No counterpart in the reference. */
int rbk_ctx_arm_tail_timeout_test(rbk_ctx* ctx, double limit_s, int withheld_cta);

/* ------------------------------------------------------------------------
 * LayerNorm
 * ------------------------------------------------------------------------ */

/* y = gamma * (x - mean) * rstd + beta, per row of [N, D] half; mean/rstd FP32
 * [N] out (biased variance, eps).  gamma/beta half [D].  D % 8 == 0, D <= 8192.
 * Replaces layer_norm_fp16_forward (src/cuda_kernels.cuh:99-101). */
int rbk_ln_fwd(rbk_ctx* ctx, void* y, float* mean, float* rstd, const void* x, const void* gamma,
               const void* beta, int N, int D, float eps, void* stream);

#define RBK_LN_REFERENCE_FORMULA 1  /* dx as src/cpu_mat.h:146 (one rstd factor short) */

/* LayerNorm backward over [N, D] half.
 *   dx      = dres + LN'(dy)      (dres optional: the residual-stream branch)
 *   dgamma += sum_rows dy * xhat,  dbeta += sum_rows dy        (FP32 [D])
 *   dbias_out (optional) += sum_rows dx  (FP32 [D]; the bias gradient of the
 *            linear layer whose output is this residual stream)
 * dx is the exact gradient unless flags has RBK_LN_REFERENCE_FORMULA.
 * Column sums are reduced deterministically through ctx scratch.
 * Replaces layer_norm_fp16_backward (src/cuda_kernels.cuh:102-104). */
int rbk_ln_bwd(rbk_ctx* ctx, void* dx, float* dgamma, float* dbeta, float* dbias_out, const void* dy,
               const void* dres, const void* x, const void* gamma, const float* mean, const float* rstd,
               int N, int D, int flags, void* stream);

/* rbk_ln_bwd for callers that cannot allocate device memory: no rbk_ctx, no
 * cudaMalloc / cudaFree or allocating library call.  No counterpart in the
 * reference.  Meant for hosts whose device memory is all owned by their own
 * pool (as the reference trainer's fixed MemPool arena) or that cannot take
 * the device-wide synchronisation an allocation costs inside a step loop.
 * Same arguments and outputs as rbk_ln_bwd; it runs a different kernel (the
 * non-ring LayerNorm backward), so the results agree with rbk_ln_bwd to
 * rounding, not bit for bit.
 *   - Scratch: one fixed array of RBK_LN_BWD_NOALLOC_SCRATCH_BYTES (4 MiB) in
 *     device memory, reserved once by every GPU that loads the library and
 *     held until the process exits; enough for D <= 2048 on a 148-SM B200.
 *     Larger needs are rejected with RBK_ERR_INVALID (use rbk_ln_bwd).
 *   - The first call on each device looks up that array's device address
 *     (with the device current); make that first call before any stream
 *     capture.  `stream` must belong to the current device (RBK_ERR_INVALID
 *     otherwise).
 *   - Every call shares the one array.  Each call overwrites the whole part it
 *     uses, so nothing carries over, but calls that overlap on the GPU (other
 *     streams, other threads) race on it: serialise them. */
#define RBK_LN_BWD_NOALLOC_SCRATCH_BYTES (4u << 20)
int rbk_ln_bwd_noalloc(void* dx, float* dgamma, float* dbeta, float* dbias_out, const void* dy, const void* dres,
                       const void* x, const void* gamma, const float* mean, const float* rstd, int N, int D,
                       int flags, void* stream);

/* ------------------------------------------------------------------------
 * Softmax cross-entropy (LM head loss)
 * ------------------------------------------------------------------------ */

/* One pass over half logits [N, V] (row stride ld >= V, ld % 8 == 0,
 * V <= 65536):
 *   dlogits[i, j] = (softmax(z_i)_j - [j == t_i]) * scale * (*dscale if dscale)
 * dlogits may alias logits (in place), or be NULL for a loss-only pass.  Output:
 *   row_loss [N] FP32 = -log(softmax(z_i)_{t_i} + 1e-10)  (src/cpu_mat.h:213)
 * A target outside [0, V) yields a NaN row loss and a zero gradient row.
 * The lm_b gradient (column sums of dlogits) comes from the LM-head wgrad
 * (rbk_gemm_desc.dbias_rows), which reads dlogits anyway.
 * `scale` carries the 1/N of the mean (src/cpu_mat.h:233) and any upstream
 * factor; dscale (device FP32, optional) is the dynamic loss scale.
 * Replaces cross_entropy_fp32_forward/_backward (src/cuda_kernels.cuh:127-128)
 * and the scale_add that follows them (src/model.cu:348-350). */
int rbk_softmax_xent_bwd(rbk_ctx* ctx, void* dlogits, const void* logits, int ld, const int* targets, int N,
                         int V, float scale, const float* dscale, float* row_loss, void* stream);

/* Sum of row_loss[0..N) * scale into *out (device FP32), deterministic. */
int rbk_sum(rbk_ctx* ctx, float* out, const float* x, int n, float scale, void* stream);

/* ------------------------------------------------------------------------
 * Attention softmax backward (materialised probabilities)
 * ------------------------------------------------------------------------ */

/* dS = P * (dP - rowsum(dP * P)) over nmat stacked [T, T] half matrices.
 * causal != 0: row i covers columns 0..i only; the strict upper triangle of
 * dS is not written.  T % 8 == 0.
 * Replaces softmax_fp16_backward / softmax_fp32_backward
 * (src/cuda_kernels.cuh:120,124). */
int rbk_attn_softmax_bwd(rbk_ctx* ctx, void* dS, const void* P, const void* dP, int nmat, int T, int causal,
                         void* stream);

/* ------------------------------------------------------------------------
 * Embeddings
 * ------------------------------------------------------------------------ */

/* x[b*S+s] = tok_emb[tokens[b*S+s]] + pos_emb[s]   (half [B*S, D]).
 * Replaces embedding_fp16_forward + the pos scale_add (src/model.cu:246-248). */
int rbk_embed_fwd(rbk_ctx* ctx, void* x, const void* tok_emb, const void* pos_emb, const int* tokens, int B,
                  int S, int D, int V, void* stream);

/* dtok[tokens[i]] += dx[i] (FP32 [V, D]);  dpos[s] += sum_b dx[b*S+s]
 * (FP32 [S, D]).  Either output may be NULL.
 * Replaces embedding_fp16_backward (src/cuda_kernels.cuh:112) and adds the
 * pos_emb gradient the reference never computes. */
int rbk_embed_bwd(rbk_ctx* ctx, float* dtok, float* dpos, const void* dx, const int* tokens, int B, int S,
                  int D, int V, void* stream);

/* ------------------------------------------------------------------------
 * Mixed-precision tail
 * ------------------------------------------------------------------------ */

/* Dynamic loss-scaler state, resident in device memory (LossScaler,
 * src/cuda_kernels.cuh:62-73; backoff 0.5, growth 2.0, clamp [1, 65536]). */
typedef struct rbk_scaler {
    float scale;          /* current loss scale                                 */
    int unskipped;        /* clean steps since the last growth / overflow       */
    int interval;         /* growth interval (2000)                             */
    int skipped;          /* 1 when the last tail call skipped its update       */
    int applied_steps;    /* updates applied so far (Adam's t when t <= 0)       */
    int overflow_steps;   /* total skipped steps                                */
    int status;           /* 0, or RBK_ERR_TIMEOUT from the tail's grid barrier */
    int pad;
} rbk_scaler;

typedef struct rbk_tail_args {
    float* p32;              /* FP32 masters [n]                                  */
    float* g;                /* FP32 gradients [n] (scaled by scaler.scale); zeroed */
    float* m;                /* Adam first moment [n]                             */
    float* v;                /* Adam second moment [n]                            */
    void* p16;               /* half copy of the masters [n] (may be NULL)        */
    int64_t n;
    /* Optional per-tensor L2 clip (src/model.cu:493-523) of the unscaled
     * gradients: nseg tensors [seg_off[i], seg_off[i] + seg_len[i]) (host
     * arrays).  max_norm <= 0 disables clipping. */
    const int64_t* seg_off;
    const int64_t* seg_len;
    int nseg;
    float max_norm;
    float lr, beta1, beta2, eps, weight_decay;
    int t;                   /* 1-based Adam step; <= 0: scaler->applied_steps + 1 */
    rbk_scaler* scaler;      /* device pointer                                    */
} rbk_tail_args;

/* One kernel: inf/NaN check of every gradient, unscale by 1/scale, optional
 * per-tensor clip, L2-coupled AdamW (src/cpu_mat.h:280-292), FP16 copy-out,
 * gradient zeroing, loss-scaler update and the skip decision.  On overflow the
 * masters and moments are left untouched and the step is skipped.
 * Replaces check_overflow_all (src/cuda_kernels.cu:1060-1074),
 * update_loss_scale (src/model.cu:436-449), optimizer_step (src/model.cu:454-488),
 * clip_gradients (src/model.cu:493-523) and convert_fp32_to_fp16
 * (src/cuda_kernels.cuh:186). */
int rbk_adam_tail(rbk_ctx* ctx, const rbk_tail_args* args, void* stream);

/* ------------------------------------------------------------------------
 * GEMM (tcgen05 / TMEM, TMA-fed)
 * ------------------------------------------------------------------------ */

enum {
    RBK_EPI_STORE_F16 = 0,  /* C16 = alpha*acc [+ bias[n]] [+ aux[m,n]]              */
    RBK_EPI_BIAS_GELU = 1,  /* C16 = acc + bias[n] (pre-activation); aux_out16 = gelu;
                               C may be NULL: only the activation is stored        */
    RBK_EPI_GELU_BWD = 2,   /* C16 = acc * gelu'(aux[m,n])                           */
    RBK_EPI_ACC_F32 = 3,    /* C32[m,n] += alpha*acc   (gradient accumulation)       */
    RBK_EPI_STORE_F32 = 4   /* C32[m,n] = alpha*acc                                  */
};

/* C[M,N] = op(A)[M,K] . op(B)[N,K]^T in FP32 on the tensor cores, half inputs.
 *   a_major 0: A(m,k) = A[m*lda + k] (K-major);  1: A(m,k) = A[k*lda + m]
 *   b_major 0: B(n,k) = B[n*ldb + k] (K-major);  1: B(n,k) = B[k*ldb + n]
 *   C(m,n) = C[m*ldc + n]; aux/aux_out share ldc unless ld_aux is given.
 * Leading dimensions must be multiples of 8 elements and base pointers
 * 16-byte aligned (TMA).  split_k 0 = automatic (only for RBK_EPI_ACC_F32).
 * Replaces gemm_fp16_tensorcores, gemm_fp16_accum_fp32 and its _backward_dA /
 * _backward_dB variants, linear_forward_fp16(_to_fp32) and linear_backward_fp16
 * (src/cuda_kernels.cuh:137-147,190-193), plus the FFN/QKV fusions
 * (src/cuda_kernels.cuh:153-169). */
typedef struct rbk_gemm_desc {
    int M, N, K;
    const void* A; int lda; int a_major;
    const void* B; int ldb; int b_major;
    void* C; int ldc;
    int epilogue;
    const void* bias;        /* half [N]                                   */
    const void* aux;         /* half [M, ld_aux]: residual or pre-activation */
    int ld_aux;              /* 0 -> ldc                                    */
    void* aux_out;           /* half [M, ld_aux]: activation output         */
    float* dbias_rows;       /* ACC_F32 only: FP32 [M] += alpha * row sums of
                                op(A) over K — the bias gradient of a linear
                                layer when A = dY^T (one extra N=16 MMA
                                against a ones tile, issued by the n = 0 tiles) */
    float alpha;
    int split_k;
} rbk_gemm_desc;

int rbk_gemm(rbk_ctx* ctx, const rbk_gemm_desc* d, void* stream);

/* Linear-layer shorthands over the [out, in] weight layout:
 *   fwd  : Y[N,out] = X[N,in] W^T (+ bias) (+ residual)      -> STORE_F16
 *   dgrad: dX[N,in] = dY[N,out] W  [* gelu'(gelu_pre)]      -> STORE_F16 or GELU_BWD
 *   wgrad: dW[out,in] += dY^T X   (FP32 accumulate)          -> ACC_F32 (+ bias grad)
 * Replaces gemm_fp16_accum_fp32_backward_dA / _dB (src/cuda_kernels.cu:639-665). */
int rbk_linear_fwd(rbk_ctx* ctx, void* Y, const void* X, const void* W, const void* bias, const void* residual,
                   int N, int in, int out, void* stream);
int rbk_gemm_dgrad(rbk_ctx* ctx, void* dX, const void* dY, const void* W, int N, int in, int out,
                   const void* gelu_pre, void* stream);
/* dbias (optional, FP32 [out]) += column sums of dY, fused into the wgrad. */
int rbk_gemm_wgrad(rbk_ctx* ctx, float* dW, float* dbias, const void* dY, const void* X, int N, int in, int out,
                   void* stream);

/* ------------------------------------------------------------------------
 * LoRA adapters, kernel level (the model level runs the same GEMMs inside
 * rbk_model_forward / _backward once rbk_model_lora_enable has been called)
 * ------------------------------------------------------------------------ */

/* One adapter on one projection, W' = W + scaling A B, A [in, r] and B [r, out]
 * row-major FP16 (the per-target step of lora_forward_all, src/lora.h:224-226):
 *   xa[N, r] = x A   (FP16, kept for the backward);   y[N, out] += scaling xa B
 * x, y FP16 with row strides ldx, ldy (y updated in place, e.g. the q or v
 * columns of a fused qkv).  in, out, r and the strides are multiples of 8. */
int rbk_lora_fwd(rbk_ctx* ctx, void* y, int ldy, void* xa, const void* x, int ldx, const void* A, const void* B,
                 int N, int in, int r, int out, float scaling, void* stream);
/* Its backward (lora_backward_all, src/lora.h:227-229):
 *   dB[r, out] += scaling xa^T dy;   dyb[N, r] = scaling dy B^T (caller's FP16
 *   workspace);   dA[in, r] += x^T dyb;   dx[N, in] += dyb A^T (FP16, in place,
 *   row stride lddx; NULL skips it).  dA, dB FP32. */
int rbk_lora_bwd(rbk_ctx* ctx, float* dA, float* dB, void* dx, int lddx, void* dyb, const void* dy, int lddy,
                 const void* x, int ldx, const void* xa, const void* A, const void* B, int N, int in, int r, int out,
                 float scaling, void* stream);
/* lora_optimizer_step (src/lora.h:230): the fused AdamW tail (rbk_adam_tail)
 * over an adapter arena: FP32 masters / grads / moments, the FP16 copy the
 * adapter GEMMs read, the shared loss scaler. */
int rbk_lora_adam(rbk_ctx* ctx, const rbk_tail_args* args, void* stream);

/* ------------------------------------------------------------------------
 * Causal flash attention (d_head 64 or 128)
 * ------------------------------------------------------------------------ */

/* qkv: half [B*S, 3*H*dh] with q | k | v column blocks (the fused QKV GEMM
 * output); o: half [B*S, H*dh]; lse: FP32 [B, H, S] (natural-log sum-exp of
 * the scaled scores).  scale = 1/sqrt(dh) (src/cpu_model.cpp:148).
 * Replaces the per-(b,h) score GEMMs, apply_causal_mask_fp32 and
 * softmax_fp32_forward of src/model.cu:262-286. */
int rbk_attn_fwd(rbk_ctx* ctx, void* o, float* lse, const void* qkv, int B, int S, int H, int dh, float scale,
                 void* stream);

/* dqkv: half [B*S, 3*H*dh] (dq | dk | dv); dbias_qkv (optional) FP32 [3*H*dh]
 * += column sums of dqkv (the bq | bk | bv gradients).  The reference never
 * runs an attention backward (src/model.cu:387-397 sets dQ = dK = dV = dO). */
int rbk_attn_bwd(rbk_ctx* ctx, void* dqkv, float* dbias_qkv, const void* qkv, const void* o, const void* dout,
                 const float* lse, int B, int S, int H, int dh, float scale, void* stream);

/* ------------------------------------------------------------------------
 * Model: the RubidiumTransformer drop-in (src/model.h:112-139)
 * ------------------------------------------------------------------------ */

typedef struct rbk_model rbk_model;

typedef struct rbk_model_opts {
    int max_batch;                     /* B of allocate_activations(B*T)            */
    int max_seq;                       /* S <= cfg.T                                */
    int use_activation_checkpointing;  /* ModelConfig field, src/model.h:19         */
    float init_loss_scale;             /* 65536 (src/model.h:120)                   */
    int growth_interval;               /* 2000                                      */
    int device;
} rbk_model_opts;

/* Buffer families of the parameter arena (include/rbk_layout.h), plus the
 * model's device loss scalar (FP32, n = 1) and its logits / dlogits buffer
 * (half [max_batch * max_seq, round_up(V, 8)]). */
enum { RBK_BUF_P16 = 0, RBK_BUF_P32 = 1, RBK_BUF_GRAD = 2, RBK_BUF_M = 3, RBK_BUF_V = 4,
       RBK_BUF_LOSS = 5, RBK_BUF_LOGITS = 6 };

int rbk_model_create(rbk_model** out, const rbk_config* cfg, const rbk_model_opts* opts);
int rbk_model_destroy(rbk_model* m);
/* The model's own context (for rbk_ctx_profile / rbk_ctx_device_error). */
int rbk_model_ctx(rbk_model* m, rbk_ctx** ctx);
/* Device pointer and element count of one arena family. */
int rbk_model_buffer(rbk_model* m, int which, void** ptr, int64_t* n);
/* Device pointer to the loss scaler state (rbk_scaler). */
int rbk_model_scaler(rbk_model* m, rbk_scaler** dev);
/* Copy FP32 masters to the FP16 weights (convert_weights_fp32_to_fp16, src/model.h:129). */
int rbk_model_sync_fp16(rbk_model* m, void* stream);
/* init_weights (src/model.cu:146-183): seeded N(0, std) matrices and
 * embeddings, LN gamma 1 / beta 0, biases 0; zero moments and gradients. */
int rbk_model_init_weights(rbk_model* m, uint64_t seed, float std, void* stream);
/* save / load (src/model.h:136-137, src/model.cu:585-679).  The file starts
 * with the reference's RBN2 layout: "RBN2", V T D H L FF (int32), a 256-entry
 * int32 character map (char_map, or zeros when NULL), then every FP16 weight
 * in the reference's tensor order (token_emb, pos_emb; per layer ln1_w ln1_b
 * ln2_w ln2_b wq bq wk bk wv bv wo bo w1 b1 w2 b2; ln_f_w ln_f_b lm_w lm_b),
 * rows * cols elements each.  An extension block follows that the reference
 * loader never reads: "RBKX", version 1 (int32), the element count of one
 * family (int64), the rbk_scaler state, then the FP32 masters, Adam m and
 * Adam v in the same order.  The reference passes device pointers to
 * fwrite / fread and keeps no optimizer state; here a resumed run continues
 * Adam and the loss-scale schedule exactly.  Both calls synchronise `stream`
 * first.  load requires the file's config to equal the model's
 * (RBK_ERR_INVALID otherwise); a file without the extension block (the
 * reference's own) loads with masters = FP32(FP16 weights), zero moments and
 * a fresh scaler.  Gradients are zeroed.  File errors return RBK_ERR_IO.
 * LoRA adapters and their moments are not part of the file (the base model
 * and its optimizer state are). */
/* The trainer loop of src/main.cpp:125-175 on the device.  For each of
 * `steps` steps (numbered first_step, first_step + 1, ...): `ga` micro-steps,
 * each gathering B windows of T + 1 tokens from the device-resident token
 * stream (tokens = stream[o + t], targets = stream[o + t + 1]), forward,
 * backward with grad_scale (the reference passes 1/(B*ga), src/main.cpp:158);
 * then the optimizer step with the reference's LR schedule (linear warm-up
 * over `warmup` steps, then cosine to 0 at max_steps, src/main.cpp:127-131)
 * and per-tensor clip `clip` (0: none); with LoRA enabled, the LoRA step
 * (src/fine_tune.cu) instead.  Window starts come from `starts` (host,
 * [steps * ga * B], each in [0, n_tokens - T - 1], uploaded once) or, when
 * NULL, from a SplitMix64 hash of (seed, run-wide sample index), so a run
 * resumed at first_step draws the windows it would have drawn.  The reference
 * instead cudaMallocs and blocking-copies every micro-batch, reads every loss
 * back and synchronises the device every step; this call enqueues the whole
 * run and synchronises once, to read the losses back when `losses` (host,
 * [steps], the mean over ga of the micro-step losses) is non-NULL.  Its
 * buffers are stream-ordered allocations (cudaMallocAsync). */
typedef struct rbk_train_args {
    const int* tokens;       /* device int32 token stream [n_tokens]          */
    int64_t n_tokens;
    const int64_t* starts;   /* host window starts, or NULL (device-drawn)     */
    uint64_t seed;
    int steps, ga, B, T;
    int first_step;          /* >= 1; Adam's t and the LR schedule's step       */
    int max_steps, warmup;
    float lr, b1, b2, eps, wd, clip;
    float grad_scale;
    float* losses;           /* host [steps] or NULL                           */
} rbk_train_args;
int rbk_model_train(rbk_model* m, const rbk_train_args* a, void* stream);
int rbk_model_save(rbk_model* m, const char* path, const int* char_map, void* stream);
int rbk_model_load(rbk_model* m, const char* path, int* char_map_out, void* stream);


/* forward (src/model.h:130): device tokens/targets [B*S] int32.  Writes the
 * mean loss to *loss_dev (device FP32) when non-NULL; targets may be NULL.
 * In training mode (the default) the pass that computes the loss also writes
 * dlogits over the logits buffer for the following backward; in eval mode
 * (rbk_model_set_training(m, 0)) the logits are left intact and backward
 * recomputes dlogits from them. */
int rbk_model_forward(rbk_model* m, const int* tokens, const int* targets, int B, int S, float* loss_dev,
                      void* stream);
/* backward (src/model.h:131): accumulates gradients of
 *   loss * grad_scale * scaler.scale
 * into the gradient arena (grad_scale is the reference's loss_scale argument,
 * 1/(BS*GA) in src/main.cpp:158; pass 1 for the plain mean).  Must follow a
 * forward on the same tokens.  The arena is the library's between calls: while
 * it is known to hold zeros (after rbk_model_create, rbk_model_init_weights,
 * rbk_model_zero_grad or an optimizer step, which zeroes it) the weight-gradient
 * GEMMs store their tiles instead of reading and adding, so values written into
 * it through rbk_model_buffer after one of those calls are overwritten, not
 * added to.  A caller that zeroes the arena itself uses rbk_model_zero_grad. */
int rbk_model_backward(rbk_model* m, const int* tokens, const int* targets, int B, int S, float grad_scale,
                       void* stream);
/* Zero the gradient arena on `stream` (what the reference's backward does at
 * entry, src/model.cu:325-340; here the optimizer step already does it). */
int rbk_model_zero_grad(rbk_model* m, void* stream);
/* Training (1, default) / eval (0) mode, see rbk_model_forward. */
int rbk_model_set_training(rbk_model* m, int training);
/* optimizer_step (src/model.h:132) fused with the overflow check, unscale,
 * optional per-tensor clip (max_norm <= 0: off), scaler update and skip. */
int rbk_model_optimizer_step(rbk_model* m, int t, float lr, float b1, float b2, float eps, float wd,
                             float max_norm, void* stream);

/* ------------------------------------------------------------------------
 * LoRA (src/lora.h:13-231): rank-r adapters on the Q and V projections.
 * ------------------------------------------------------------------------ */

/* Enable adapters: A [L, D, r] ~ N(0, 0.02) (seeded), B [L, r, D] = 0,
 * scaling alpha / r.  Base weights become frozen: backward produces only the
 * adapter gradients (plus the dgrads through the frozen base).
 * Replaces init_lora (src/lora.h:223). */
int rbk_model_lora_enable(rbk_model* m, int rank, float alpha, uint64_t seed, void* stream);
/* Device pointers of the adapter arenas: which = RBK_BUF_P32 (A|B masters),
 * RBK_BUF_GRAD, RBK_BUF_M, RBK_BUF_V.  Layout: Aq [L,D,r] | Bq [L,r,D] |
 * Av [L,D,r] | Bv [L,r,D]. */
int rbk_model_lora_buffer(rbk_model* m, int which, void** ptr, int64_t* n);
/* lora_optimizer_step (src/lora.h:230) with the same fused tail. */
int rbk_model_lora_step(rbk_model* m, int t, float lr, float b1, float b2, float eps, float wd, void* stream);
/* Overflow injection for testing the skip path: before the next backward's
 * LM-head dgrad, set every `stride`-th element of dlogits (starting at
 * `offset`) to +inf.  stride <= 0 disables. */
int rbk_model_inject_inf(rbk_model* m, int64_t offset, int64_t stride);

/* ------------------------------------------------------------------------
 * Data parallel: bucketed NCCL all-reduce of the gradient arena, overlapped
 * with the backward (no counterpart in the reference, which is single-GPU:
 * src/main.cpp:54).
 * ------------------------------------------------------------------------ */

#define RBK_NCCL_ID_BYTES 128
/* The all-reduce schedule (host only, no GPU needed): *count buckets, each
 * out[3i..3i+2] = {backward unit after which it is launched (0 = LN_f + LM
 * head, 1..L = layers L-1..0, L+1 = embeddings), arena begin, arena end}.
 * Buckets tile the arena exactly once, in descending address order. */
int rbk_dp_plan(const rbk_config* cfg, int64_t bucket_bytes, int64_t* out, int max, int* count);
/* Fill a 128-byte NCCL unique id on the root rank (ncclGetUniqueId). */
int rbk_dp_unique_id(void* id128);
/* Join the communicator; bucket_bytes (25 MB) sets the all-reduce granularity.
 * Defaults of rbk_model_dp_init_ex, overridable through the environment:
 * RBK_NCCL_MAX_CTAS (0), RBK_NCCL_TIMEOUT_S (300), RBK_DP_SHARD (0). */
int rbk_model_dp_init(rbk_model* m, const void* id128, int rank, int world, int64_t bucket_bytes);
typedef struct rbk_dp_opts {
    int64_t bucket_bytes;   /* all-reduce granularity (25 MB)                            */
    int max_ctas;           /* NCCL CTA cap for the buckets that overlap the backward, so
                               NCCL leaves SMs to the GEMM grids (0: NCCL's default); the
                               last bucket, reduced after the backward, is not capped  */
    double timeout_s;       /* watchdog deadline per collective (<= 0: 300 s)            */
    int shard_optimizer;    /* 1: sharded optimizer.  Each bucket is reduce-scattered (not
                               all-reduced): rank r receives the summed gradients of the r-th
                               1/world slice of every bucket and runs the optimizer tail on
                               those slices only; the updated FP16 weights are all-gathered
                               bucket by bucket, overlapped with the next forward, which waits
                               for each bucket before its first use.  FP32 masters and Adam
                               moments then hold this rank's slices only until
                               rbk_model_dp_gather_state (called by rbk_model_save and
                               rbk_model_sync_fp16).  Needs every bucket length to divide into
                               world slices of a multiple of 4 elements (world = 1, 2, 4, 8, 16).
                               0: every rank all-reduces and updates the whole arena.          */
} rbk_dp_opts;
/* rbk_model_dp_init with explicit options.  The communicators are non-blocking
 * (ncclCommInitRankConfig, blocking = 0) and watched by a host thread: a
 * collective still incomplete after timeout_s (a peer that left, a hung link)
 * or an asynchronous NCCL error aborts them (ncclCommAbort, which ends NCCL
 * kernels waiting on a peer).  From then on rbk_model_dp_status, backward and
 * the optimizer steps return RBK_ERR_TIMEOUT / RBK_ERR_NCCL (nothing is
 * applied); the model must be shut down (rbk_model_dp_shutdown) and rebuilt. */
int rbk_model_dp_init_ex(rbk_model* m, const void* id128, int rank, int world, const rbk_dp_opts* o);
/* RBK_OK, or the status that made the watchdog abort the communicators. */
int rbk_model_dp_status(rbk_model* m);
/* Abort this rank's communicators now (local, not collective): a rank that
 * leaves the job calls it instead of a shutdown its peers would have to join;
 * afterwards the model behaves as after a watchdog abort (RBK_ERR_NCCL). */
int rbk_model_dp_abort(rbk_model* m);
/* Kernel-level data parallelism for callers that keep their own orchestration
 * (no rbk_model): the same non-blocking communicators, high-priority
 * communication stream and watchdog as rbk_model_dp_init_ex (opts: max_ctas,
 * timeout_s; NULL for the defaults; bucket_bytes and shard_optimizer unused).
 * rbk_dp_init makes `device` the calling thread's current device.
 *   rbk_dp_bucket_ready: sum-all-reduce buf[0, n) FP32 in place over the ranks,
 *     on the communication stream, after the work enqueued on `stream` so far
 *     (call it as soon as a bucket's gradients are final; it overlaps what
 *     follows on `stream`);
 *   rbk_dp_finish: `stream` waits for every bucket enqueued so far;
 *   rbk_dp_status / rbk_dp_abort / rbk_dp_destroy: as the rbk_model_dp_* ones.
 * No counterpart in the reference (single GPU, src/main.cpp:54). */
typedef struct rbk_dp rbk_dp;
int rbk_dp_init(rbk_dp** out, int device, const void* id128, int rank, int world, const rbk_dp_opts* opts);
int rbk_dp_bucket_ready(rbk_dp* dp, float* buf, int64_t n, void* stream);
int rbk_dp_finish(rbk_dp* dp, void* stream);
int rbk_dp_status(rbk_dp* dp);
int rbk_dp_abort(rbk_dp* dp);
int rbk_dp_destroy(rbk_dp* dp);
/* Sharded optimizer: *count = number of [begin, end) arena ranges this rank
 * updates (0 when not sharded); out[2i], out[2i+1] = range i, for i < max. */
int rbk_model_dp_shard_ranges(rbk_model* m, int64_t* out, int max, int* count);
/* Sharded optimizer: all-gather the FP32 masters and Adam moments on `stream`
 * so every rank holds all of them again (a no-op when they are whole). */
int rbk_model_dp_gather_state(rbk_model* m, void* stream);
/* Gradient accumulation under data parallelism (the reference accumulates GA
 * micro-steps per optimizer step, src/main.cpp:136-164).  sync = 0: following
 * backwards only accumulate this rank's gradients, no all-reduce; sync = 1
 * (the default): backward all-reduces the whole accumulated arena bucket by
 * bucket.  Set 0 before the first GA - 1 micro-steps of a step and 1 before
 * the last; rbk_model_train does this itself.  Each rank's micro-steps then
 * enter the reduced sum exactly once. */
int rbk_model_dp_set_sync(rbk_model* m, int sync);
int rbk_model_dp_shutdown(rbk_model* m);

/* ------------------------------------------------------------------------
 * GPU BPE tokenizer (src/tokenizer_cuda.h:120-164, src/tokenizer_cuda.cu:90-348)
 * ------------------------------------------------------------------------
 * Special ids as the reference's: PAD 0, UNK 1, BOS 2, EOS 3, SEP 4; byte c
 * encodes as c + 5.  A pair merges into the result of the first rule, in
 * rule order, with that pair; merges run in greedy left-to-right passes until
 * a pass merges nothing; EOS ends every row.  Results equal the reference's
 * encode_kernel / decode_kernel wherever those are defined; the contract
 * where they are not is stated at each call.  A handle serves one device and
 * one host thread at a time. */
typedef struct rbk_bpe rbk_bpe;
/* tokenizer_copy_to_device / tokenizer_init_gpu (src/tokenizer_cuda.cu:205-272,
 * 391-394).  The tables are the ones the reference's builders produce:
 *   inverse vocabulary: id i's string is inv_bytes[inv_offsets[i] ..
 *     + inv_lengths[i]) for i < vocab_size (build_inv_vocab_arrays, :488-505);
 *   merge rules in merge order: (merge_first[j], merge_second[j]) ->
 *     merge_result[j] (the rules array of build_merge_trie, :408-454).
 * vocab_size >= 261 (specials + bytes); results inside the vocabulary.  A
 * rule whose pair holds an id outside [0, vocab_size) can never fire and is
 * dropped; a repeated pair keeps its first rule.  Fails with
 * RBK_ERR_UNSUPPORTED on a device other than sm_100. */
int rbk_bpe_create(rbk_bpe** out, int device, int vocab_size, const char* inv_bytes, int64_t inv_bytes_size,
                   const int* inv_offsets, const int* inv_lengths, const int* merge_first, const int* merge_second,
                   const int* merge_result, int num_merges);
/* tokenizer_free_gpu (:274-285).  Waits for the handle's staging copies. */
int rbk_bpe_destroy(rbk_bpe* t);
/* Distinct rules the handle's pair table holds. */
int rbk_bpe_num_rules(const rbk_bpe* t);
/* encode_batch (src/tokenizer_cuda.cu:287-332): `batch` NUL-terminated host
 * strings -> device rows out_tokens[b * max_seq_len ..] and out_lengths[b]
 * (tokens + 1, the EOS included).  Asynchronous on `stream` (the strings may
 * be reused once the call returns).  Row b holds the tokens, EOS, then PAD up
 * to max_seq_len (the reference leaves pass scratch there).  An empty string
 * gives [EOS], length 1 (the reference writes nothing).  A string of more
 * than max_seq_len - 1 bytes is rejected with RBK_ERR_INVALID before anything
 * runs (the reference writes past its row); one of exactly max_seq_len - 1
 * bytes is merged like any other (the reference skips its merges).
 * 2 <= max_seq_len <= 8193.  Large batches (>= 4096 strings, >= 8 MiB of text) are
 * staged and encoded in four parts, each part's copy and launch overlapping the host
 * packing of the next. */
int rbk_bpe_encode_batch(rbk_bpe* t, const char* const* strings, int batch, int* out_tokens, int* out_lengths,
                         int max_seq_len, void* stream);
/* The same encode over strings already on the device: string b is
 * bytes[offsets[b] .. offsets[b] + lengths[b]) (any byte values, NUL
 * included).  A string longer than max_seq_len - 1 bytes is cut to its first
 * max_seq_len - 1 bytes and counted into *n_truncated (device int, may be
 * NULL). */
int rbk_bpe_encode(rbk_bpe* t, const uint8_t* bytes, const int64_t* offsets, const int* lengths, int batch,
                   int* out_tokens, int* out_lengths, int max_seq_len, int* n_truncated, void* stream);
/* decode_batch (src/tokenizer_cuda.cu:334-348): device token rows -> device
 * strings out[b * max_string_len ..], NUL-terminated, the bytes after the NUL
 * untouched.  Row b has lengths[b] tokens; rows sit ld tokens apart (at most
 * ld read), or with ld == 0 row b starts at b * lengths[b] as in the
 * reference (:182).  A token id outside [0, vocab_size) adds no bytes and is
 * counted into *n_bad (device int, may be NULL); the reference reads outside
 * its tables there. */
int rbk_bpe_decode_batch(rbk_bpe* t, const int* tokens, int64_t ld, const int* lengths, int batch, char* out,
                         int max_string_len, int* n_bad, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* RBK_H */
