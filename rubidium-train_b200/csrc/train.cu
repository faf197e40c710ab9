// train.cu — the reference's trainer loop (src/main.cpp:125-175) with the
// training data resident on the device and no host synchronisation per step.
//
// The reference samples BS random windows of the token stream on the host for
// every micro-step, cudaMallocs two buffers, copies the windows over with
// blocking cudaMemcpy, runs forward (which returns the loss to the host, a
// synchronisation), backward, cudaFrees, and ends each step with
// cudaDeviceSynchronize.  Here the token stream is uploaded once by the
// caller; a gather kernel builds each micro-batch (tokens = stream[o + t],
// targets = stream[o + t + 1]) from window starts that are either given for the
// whole run (uploaded once) or drawn on the device from a seed; losses
// accumulate in a device array; the LR schedule is evaluated on the host and
// passed by value.  The only synchronisation is the read-back of the losses at
// the end (none when the caller does not want them).
#include <cmath>
#include <vector>

#include "common.cuh"
#include "model.h"

namespace rbk {
namespace {

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// tok[b, t] = stream[o_b + t], tgt[b, t] = stream[o_b + t + 1] with o_b = starts[b], or, without
// starts, a SplitMix64 draw of (seed, sample0 + b) in [0, n - T - 1).
__global__ void gather_windows_kernel(int* __restrict__ tok, int* __restrict__ tgt, const int* __restrict__ stream,
                                      int64_t n, const int64_t* __restrict__ starts, uint64_t seed, int64_t sample0,
                                      int B, int T) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * T) return;
    const int b = i / T, t = i - b * T;
    int64_t o;
    if (starts) {
        o = starts[b];
    } else {
        const uint64_t r = splitmix64(seed ^ splitmix64((uint64_t)(sample0 + b)));
        o = (int64_t)(r % (uint64_t)(n - T - 1));
    }
    tok[i] = stream[o + t];
    tgt[i] = stream[o + t + 1];
}

// src/main.cpp:127-131
float lr_at(const rbk_train_args* a, int step) {
    if (step < a->warmup) return a->lr * (float)step / (float)a->warmup;
    const float p = a->max_steps > a->warmup ? (float)(step - a->warmup) / (float)(a->max_steps - a->warmup) : 0.0f;
    return a->lr * 0.5f * (1.0f + cosf(3.14159265f * p));
}

}  // namespace
}  // namespace rbk

using namespace rbk;

extern "C" int rbk_model_train(rbk_model* m, const rbk_train_args* a, void* stream) {
    RBK_REQUIRE(m && a && a->tokens, "rbk_model_train: null pointer");
    RBK_REQUIRE(a->steps > 0 && a->ga > 0 && a->B > 0 && a->T > 0, "rbk_model_train: steps, ga, B, T must be > 0");
    RBK_REQUIRE(a->B <= m->opts.max_batch && a->T <= m->opts.max_seq && a->T % 64 == 0,
                "rbk_model_train: need B <= max_batch, T <= max_seq, T %% 64 == 0 (B=%d T=%d)", a->B, a->T);
    RBK_REQUIRE(a->n_tokens > (int64_t)a->T + 1, "rbk_model_train: the token stream must exceed T + 1 tokens");
    RBK_REQUIRE(a->first_step >= 1 && a->warmup >= 0, "rbk_model_train: first_step >= 1, warmup >= 0");
    const int64_t micro = (int64_t)a->steps * a->ga;
    const int64_t nstart = micro * a->B;
    if (a->starts) {
        for (int64_t i = 0; i < nstart; ++i)
            RBK_REQUIRE(a->starts[i] >= 0 && a->starts[i] <= a->n_tokens - a->T - 1,
                        "rbk_model_train: window start %lld at index %lld is outside [0, n_tokens - T - 1]",
                        (long long)a->starts[i], (long long)i);
    }
    RBK_CUDA(cudaSetDevice(m->ctx->device));
    cudaStream_t st = as_stream(stream);
    const int BT = a->B * a->T;
    // stream-ordered allocations: no device-wide synchronisation
    int *tok = nullptr, *tgt = nullptr;
    float* losses = nullptr;
    int64_t* starts = nullptr;
    RBK_CUDA(cudaMallocAsync((void**)&tok, sizeof(int) * 2 * (size_t)BT, st));
    tgt = tok + BT;
    RBK_CUDA(cudaMallocAsync((void**)&losses, sizeof(float) * (size_t)micro, st));
    if (a->starts) {
        RBK_CUDA(cudaMallocAsync((void**)&starts, sizeof(int64_t) * (size_t)nstart, st));
        RBK_CUDA(cudaMemcpyAsync(starts, a->starts, sizeof(int64_t) * (size_t)nstart, cudaMemcpyHostToDevice, st));
    }
    int rc = RBK_OK;
    const bool lora = m->lora.rank > 0;
    // Data parallel: the micro-steps before the last of each step only accumulate this rank's
    // gradients; the last one all-reduces the accumulated sum (src/main.cpp:136-164 runs GA
    // micro-steps per optimizer step).
    const bool sync_saved = m->dp.sync;
    for (int s = 0; s < a->steps && rc == RBK_OK; ++s) {
        const int step = a->first_step + s;
        for (int g = 0; g < a->ga && rc == RBK_OK; ++g) {
            m->dp.sync = g == a->ga - 1;
            const int64_t k = (int64_t)s * a->ga + g;                 // micro-step of this call
            const int64_t sample0 = ((int64_t)(step - 1) * a->ga + g) * a->B;   // run-wide sample index
            gather_windows_kernel<<<(BT + 255) / 256, 256, 0, st>>>(tok, tgt, a->tokens, a->n_tokens,
                                                                    starts ? starts + k * a->B : nullptr, a->seed,
                                                                    sample0, a->B, a->T);
            cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) { rc = cuda_fail(e, "gather_windows_kernel", __FILE__, __LINE__); break; }
            count_launch();
            rc = rbk_model_forward(m, tok, tgt, a->B, a->T, losses + k, stream);
            if (rc == RBK_OK) rc = rbk_model_backward(m, tok, tgt, a->B, a->T, a->grad_scale, stream);
        }
        if (rc != RBK_OK) break;
        const float lr = lr_at(a, step);
        rc = lora ? rbk_model_lora_step(m, step, lr, a->b1, a->b2, a->eps, a->wd, stream)
                  : rbk_model_optimizer_step(m, step, lr, a->b1, a->b2, a->eps, a->wd, a->clip, stream);
    }
    m->dp.sync = sync_saved;
    std::vector<float> h;
    if (rc == RBK_OK && a->losses) {
        h.resize((size_t)micro);
        cudaError_t e = cudaMemcpyAsync(h.data(), losses, sizeof(float) * (size_t)micro, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) rc = cuda_fail(e, "rbk_model_train: loss read-back", __FILE__, __LINE__);
    }
    cudaFreeAsync(tok, st);
    cudaFreeAsync(losses, st);
    if (starts) cudaFreeAsync(starts, st);
    if (rc == RBK_OK && a->losses) {
        for (int s = 0; s < a->steps; ++s) {
            double acc = 0.0;
            for (int g = 0; g < a->ga; ++g) acc += h[(size_t)s * a->ga + g];
            a->losses[s] = (float)(acc / a->ga);
        }
    }
    return rc;
}
