// common.cuh — shared host/device helpers of librbk (sm_100a only).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <utility>
#include <vector>

#include "rbk.h"

// ----------------------------------------------------------------------------
// Host-side error plumbing: every entry point returns an int status and leaves
// a message in a thread-local buffer (rbk_last_error).
// ----------------------------------------------------------------------------
namespace rbk {

void set_error(const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what, const char* file, int line);
void count_launch();   // every kernel launched by librbk is counted (rbk_launch_count)

}  // namespace rbk

#define RBK_CUDA(call)                                                              \
    do {                                                                            \
        cudaError_t e_ = (call);                                                    \
        if (e_ != cudaSuccess) return ::rbk::cuda_fail(e_, #call, __FILE__, __LINE__); \
    } while (0)

#define RBK_LAUNCHED(what)                                                          \
    do {                                                                            \
        cudaError_t e_ = cudaGetLastError();                                        \
        if (e_ != cudaSuccess) return ::rbk::cuda_fail(e_, what, __FILE__, __LINE__); \
        ::rbk::count_launch();                                                      \
    } while (0)

#define RBK_REQUIRE(cond, ...)                \
    do {                                      \
        if (!(cond)) {                        \
            ::rbk::set_error(__VA_ARGS__);    \
            return RBK_ERR_INVALID;           \
        }                                     \
    } while (0)

#define RBK_TRY(expr)                 \
    do {                              \
        int s_ = (expr);              \
        if (s_ != RBK_OK) return s_;  \
    } while (0)

// ----------------------------------------------------------------------------
// Context: device + scratch arena + a small zeroed area for tickets/flags.
// ----------------------------------------------------------------------------
// Optional per-category kernel timing (CUDA events around each entry point).
struct rbk_prof {
    bool on = false;
    std::vector<cudaEvent_t> pool;     // start/stop pairs
    struct Rec { int cat; double work; int sub; };   // sub: GEMM role (0 fwd, 1 dgrad, 2 wgrad) or -1
    std::vector<Rec> recs;             // recs[i] uses pool[2i], pool[2i+1]
};

struct rbk_ctx {
    int device = 0;
    int num_sms = 148;
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    // Device ints, zero at creation; each user restores its slot to zero.
    int* tickets = nullptr;
    static constexpr int kTickets = 64;
    int* err = nullptr;      // device error word written by bounded waits
    rbk_prof prof;
    // Role of the next GEMMs for the profiler (0 forward, 1 dgrad, 2 wgrad); -1: derived from
    // the descriptor (FP32-accumulating epilogues are weight gradients, an MN-major B a dgrad).
    int gemm_role = -1;
    // Set by a caller that knows the C of its next ACC_F32 GEMMs holds zeros (the model's weight
    // gradients after an optimizer step): their single-split tiles are stored, not read and added.
    int gemm_c_zero = 0;
    // Bitwise-reproducible accumulation (rbk_ctx_set_deterministic / RBK_DETERMINISTIC=1):
    // split-K weight gradients add their partial planes in split order, the attention backward
    // adds dQ in key-block order.
    int deterministic = 0;
    // One-shot test setting of the next rbk_adam_tail launch (rbk_ctx_arm_tail_timeout_test):
    // its grid-barrier wait limit in ns (0: the default kWaitTimeoutNs) and a CTA that does not
    // arrive at the barrier (-1: none).
    uint64_t test_tail_wait_ns = 0;
    int test_tail_withheld_cta = -1;
};

namespace rbk {

// Timing categories (rbk_ctx_profile_read).
enum ProfCat { kCatGemm = 0, kCatAttnFwd, kCatAttnBwd, kCatLnFwd, kCatLnBwd, kCatXent, kCatTail, kCatEmbed,
               kCatOther, kNumCats };

// Records start/stop events around one entry point when profiling is on.
struct ProfScope {
    rbk_ctx* ctx;
    cudaStream_t st;
    int idx = -1;
    ProfScope(rbk_ctx* c, cudaStream_t s, int cat, double work, int sub = -1);
    ~ProfScope();
};

// Scratch of at least `bytes` (256-byte aligned); grows (cudaFree + cudaMalloc)
// only when the current arena is too small.
int ctx_scratch(rbk_ctx* ctx, size_t bytes, void** out);

// out[c] += sum_r part[r*C + c], deterministic (ctx.cu).
int column_reduce(float* out, const float* part, int R, int C, cudaStream_t st);

// Ticket slots (see rbk_ctx::tickets).
enum TicketSlot {
    kTicketSum = 0,
    kTailOverflow = 8, kTailBarrier = 9, kTailTicket = 10, kTailTimeout = 11,
    kGemmError = 16,
    kAttnFwdTile = 20, kAttnFwdDone = 21,
};

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ------------------------------------------------ programmatic dependent launch
// A kernel launched with launch_pdl() may start while the previous kernel of its
// stream is still finishing.  It may set up shared memory, barriers and TMEM,
// but must call grid_dependency_wait() before its first global-memory access:
// that blocks until the previous kernel has completed and its writes are
// visible.  grid_dependents_launch() lets the next programmatic dependent start
// its own setup (every CTA must have called it, or exited).
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependents_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void grid_dependency_sync() {
    grid_dependency_wait();
    grid_dependents_launch();
}
// Adds the programmatic-stream-serialization attribute at attr[i] unless
// RBK_NO_PDL=1; returns the attribute count.
unsigned set_pdl(cudaLaunchAttribute* attr, unsigned i);
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = set_pdl(attr, 0);
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ----------------------------------------------------------------------------
// Device helpers
// ----------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// 8 halves <-> 8 floats through one 16-byte vector.
__device__ __forceinline__ void h8_to_f(const uint4& u, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}
__device__ __forceinline__ uint4 f_to_h8(const float* f) {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    return u;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded device-side waits give up after this long and report RBK_ERR_TIMEOUT.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;   // 2 s

// GPT-2 tanh GELU and its derivative (the FFN activation of this build; the
// reference's FFN uses ReLU, src/cpu_model.cpp:198-200).
__device__ __forceinline__ float gelu_f(float x) {
    const float c = 0.7978845608028654f, a = 0.044715f;
    return 0.5f * x * (1.0f + tanhf(c * (x + a * x * x * x)));
}
__device__ __forceinline__ float gelu_grad_f(float x) {
    const float c = 0.7978845608028654f, a = 0.044715f;
    const float t = tanhf(c * (x + a * x * x * x));
    return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * c * (1.0f + 3.0f * a * x * x);
}

}  // namespace rbk
