// ctx.cu — context, scratch arena, error strings and the small reductions
// shared by several entry points.
#include <atomic>
#include <cstring>
#include <string>

#include "common.cuh"

namespace rbk {

static thread_local char g_err[512] = "";
static std::atomic<long long> g_launches{0};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

constexpr int kProfPairs = 32768;   // ~130 timed steps of the 12-layer model

ProfScope::ProfScope(rbk_ctx* c, cudaStream_t s, int cat, double work, int sub) : ctx(c), st(s) {
    if (!c || !c->prof.on) return;
    rbk_prof& p = c->prof;
    const int i = (int)p.recs.size();
    if (i >= kProfPairs) return;
    if ((int)p.pool.size() < 2 * (i + 1)) {
        for (int k = 0; k < 2; ++k) {
            cudaEvent_t e;
            if (cudaEventCreate(&e) != cudaSuccess) return;
            p.pool.push_back(e);
        }
    }
    p.recs.push_back({cat, work, sub});
    cudaEventRecord(p.pool[2 * i], s);
    idx = i;
}

ProfScope::~ProfScope() {
    if (idx >= 0) cudaEventRecord(ctx->prof.pool[2 * idx + 1], st);
}

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int cuda_fail(cudaError_t e, const char* what, const char* file, int line) {
    set_error("%s failed: %s (%s:%d)", what, cudaGetErrorString(e), file, line);
    return e == cudaErrorMemoryAllocation ? RBK_ERR_NOMEM : RBK_ERR_CUDA;
}

int ctx_scratch(rbk_ctx* ctx, size_t bytes, void** out) {
    bytes = (bytes + 255) & ~size_t(255);
    if (bytes > ctx->scratch_bytes) {
        if (ctx->scratch) RBK_CUDA(cudaFree(ctx->scratch));
        ctx->scratch = nullptr;
        ctx->scratch_bytes = 0;
        RBK_CUDA(cudaMalloc(&ctx->scratch, bytes));
        ctx->scratch_bytes = bytes;
    }
    *out = ctx->scratch;
    return RBK_OK;
}

// out[c] += sum_r part[r*C + c]   (deterministic, fixed order over r)
__global__ void column_reduce_kernel(float* __restrict__ out, const float* __restrict__ part, int R, int C) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    float s = 0.0f;
    for (int r = 0; r < R; ++r) s += part[(size_t)r * C + c];
    out[c] += s;
}

unsigned set_pdl(cudaLaunchAttribute* attr, unsigned i) {
    static const bool off = [] {
        const char* e = getenv("RBK_NO_PDL");
        return e && e[0] == '1';
    }();
    if (off) return i;
    attr[i].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[i].val.programmaticStreamSerializationAllowed = 1;
    return i + 1;
}

int column_reduce(float* out, const float* part, int R, int C, cudaStream_t st) {
    column_reduce_kernel<<<(C + 255) / 256, 256, 0, st>>>(out, part, R, C);
    RBK_LAUNCHED("column_reduce_kernel");
    return RBK_OK;
}

// Deterministic sum of n floats into *out (times scale): one CTA per 64K-chunk
// writes a partial, the last CTA (ticket) adds the partials in order.
__global__ void sum_kernel(float* __restrict__ out, const float* __restrict__ x, int n, float scale,
                           float* __restrict__ part, int* ticket) {
    __shared__ float sw[32];
    __shared__ int last;
    const int chunk = 65536;
    const int begin = blockIdx.x * chunk, end = min(n, begin + chunk);
    float s = 0.0f;
    for (int i = begin + threadIdx.x; i < end; i += blockDim.x) s += x[i];
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) sw[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? sw[threadIdx.x] : 0.0f;
        t = warp_sum(t);
        if (threadIdx.x == 0) {
            part[blockIdx.x] = t;
            __threadfence();
            last = (atomicAdd(ticket, 1) == (int)gridDim.x - 1);
        }
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence();
        float tot = 0.0f;
        for (int b = 0; b < (int)gridDim.x; ++b) tot += ((volatile float*)part)[b];
        *out = tot * scale;
        *ticket = 0;
    }
}

}  // namespace rbk

using namespace rbk;

extern "C" {

const char* rbk_last_error(void) { return g_err; }

int rbk_version(void) { return 1; }

int rbk_ctx_create(rbk_ctx** out, int device) {
    RBK_REQUIRE(out != nullptr, "rbk_ctx_create: out is NULL");
    *out = nullptr;
    int ndev = 0;
    RBK_CUDA(cudaGetDeviceCount(&ndev));
    RBK_REQUIRE(device >= 0 && device < ndev, "rbk_ctx_create: device %d out of range (%d devices)", device, ndev);
    RBK_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    RBK_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10 || prop.minor != 0) {
        set_error("librbk is built for sm_100a (B200); device %d is sm_%d%d", device, prop.major, prop.minor);
        return RBK_ERR_UNSUPPORTED;
    }
    rbk_ctx* c = new rbk_ctx();
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    cudaError_t e = cudaMalloc(&c->tickets, sizeof(int) * (rbk_ctx::kTickets + 1));
    if (e != cudaSuccess) { delete c; return cuda_fail(e, "cudaMalloc(tickets)", __FILE__, __LINE__); }
    e = cudaMemset(c->tickets, 0, sizeof(int) * (rbk_ctx::kTickets + 1));
    if (e != cudaSuccess) { cudaFree(c->tickets); delete c; return cuda_fail(e, "cudaMemset", __FILE__, __LINE__); }
    c->err = c->tickets + rbk_ctx::kTickets;
    const char* det = getenv("RBK_DETERMINISTIC");
    c->deterministic = det && det[0] == '1';
    *out = c;
    return RBK_OK;
}

int rbk_ctx_destroy(rbk_ctx* ctx) {
    if (!ctx) return RBK_OK;
    cudaSetDevice(ctx->device);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->tickets) cudaFree(ctx->tickets);
    for (cudaEvent_t e : ctx->prof.pool) cudaEventDestroy(e);
    delete ctx;
    return RBK_OK;
}

long long rbk_launch_count(void) { return g_launches.load(); }

int rbk_ctx_profile(rbk_ctx* ctx, int enable) {
    RBK_REQUIRE(ctx, "rbk_ctx_profile: null ctx");
    ctx->prof.on = enable != 0;
    ctx->prof.recs.clear();
    // create the event pool up front so no event is created inside a timed region
    while (enable && ctx->prof.pool.size() < 2 * (size_t)kProfPairs) {
        cudaEvent_t e;
        RBK_CUDA(cudaEventCreate(&e));
        ctx->prof.pool.push_back(e);
    }
    return RBK_OK;
}

int rbk_ctx_profile_read(rbk_ctx* ctx, double* ms, double* work, int* launches, int ncat) {
    RBK_REQUIRE(ctx && ms && work && launches && ncat >= kNumCats, "rbk_ctx_profile_read: bad arguments");
    for (int c = 0; c < ncat; ++c) { ms[c] = 0.0; work[c] = 0.0; launches[c] = 0; }
    rbk_prof& p = ctx->prof;
    for (size_t i = 0; i < p.recs.size(); ++i) {
        RBK_CUDA(cudaEventSynchronize(p.pool[2 * i + 1]));
        float t = 0.0f;
        RBK_CUDA(cudaEventElapsedTime(&t, p.pool[2 * i], p.pool[2 * i + 1]));
        const int c = p.recs[i].cat;
        ms[c] += t;
        work[c] += p.recs[i].work;
        launches[c] += 1;
    }
    return RBK_OK;
}

int rbk_ctx_profile_read_gemm(rbk_ctx* ctx, double* ms, double* flops, int* launches) {
    RBK_REQUIRE(ctx && ms && flops && launches, "rbk_ctx_profile_read_gemm: bad arguments");
    for (int c = 0; c < 3; ++c) { ms[c] = 0.0; flops[c] = 0.0; launches[c] = 0; }
    rbk_prof& p = ctx->prof;
    for (size_t i = 0; i < p.recs.size(); ++i) {
        if (p.recs[i].cat != kCatGemm || p.recs[i].sub < 0 || p.recs[i].sub > 2) continue;
        RBK_CUDA(cudaEventSynchronize(p.pool[2 * i + 1]));
        float t = 0.0f;
        RBK_CUDA(cudaEventElapsedTime(&t, p.pool[2 * i], p.pool[2 * i + 1]));
        ms[p.recs[i].sub] += t;
        flops[p.recs[i].sub] += p.recs[i].work;
        launches[p.recs[i].sub] += 1;
    }
    return RBK_OK;
}

int rbk_ctx_set_deterministic(rbk_ctx* ctx, int on) {
    RBK_REQUIRE(ctx, "rbk_ctx_set_deterministic: null ctx");
    ctx->deterministic = on != 0;
    return RBK_OK;
}

int rbk_ctx_arm_tail_timeout_test(rbk_ctx* ctx, double limit_s, int withheld_cta) {
    RBK_REQUIRE(ctx, "rbk_ctx_arm_tail_timeout_test: null ctx");
    RBK_REQUIRE(limit_s >= 1e-4 && limit_s <= 2.0, "rbk_ctx_arm_tail_timeout_test: limit_s must be in [1e-4, 2]");
    RBK_REQUIRE(withheld_cta >= -1, "rbk_ctx_arm_tail_timeout_test: withheld_cta must be >= -1");
    ctx->test_tail_wait_ns = (uint64_t)(limit_s * 1e9);
    ctx->test_tail_withheld_cta = withheld_cta;
    return RBK_OK;
}

int rbk_ctx_device_error(rbk_ctx* ctx, int* status) {
    RBK_REQUIRE(ctx && status, "rbk_ctx_device_error: bad arguments");
    int v[rbk_ctx::kTickets] = {};
    RBK_CUDA(cudaMemcpy(v, ctx->tickets, sizeof(v), cudaMemcpyDeviceToHost));
    *status = v[kGemmError];
    if (v[kGemmError]) {
        const int zero = 0;
        RBK_CUDA(cudaMemcpy(ctx->tickets + kGemmError, &zero, sizeof(int), cudaMemcpyHostToDevice));
    }
    return RBK_OK;
}

int rbk_sum(rbk_ctx* ctx, float* out, const float* x, int n, float scale, void* stream) {
    RBK_REQUIRE(ctx && out && x && n > 0, "rbk_sum: bad arguments");
    const int blocks = (n + 65535) / 65536;
    void* ws;
    RBK_TRY(ctx_scratch(ctx, sizeof(float) * blocks, &ws));
    sum_kernel<<<blocks, 256, 0, as_stream(stream)>>>(out, x, n, scale, (float*)ws, ctx->tickets + kTicketSum);
    RBK_LAUNCHED("sum_kernel");
    return RBK_OK;
}

}  // extern "C"
