// xent.cu — fused softmax-cross-entropy forward + backward (HBM-bound).
//
// One CTA owns a row at a time.  Pass 1 streams the row once from HBM with
// 16-byte loads (4 in flight per thread) and keeps an online (max, sum of
// exp) per thread, merged across the CTA; pass 2 re-reads the same row — a
// few tens of KB that the CTA touched microseconds earlier, so it comes from
// L2 — and writes (softmax - onehot) * scale, in place if the caller wishes.
// DRAM therefore sees one read and one write per logit.  The number of rows in
// flight (grid x row bytes) is capped well below the 126 MB L2 so pass 2 hits.
// The reference instead rescans the whole row for every element
// (src/cuda_kernels.cu:533-551, O(N V^2)); cpuops does three passes
// (src/cpu_mat.h:220-236).  Per-row loss follows src/cpu_mat.h:213
// (-log(p_t + 1e-10)).
#include <cfloat>

#include "common.cuh"

namespace rbk {
namespace {

constexpr int kThreads = 512;
constexpr int kUnroll = 4;

// Merge two (max, sum) online-softmax states.
__device__ __forceinline__ void merge(float& m, float& s, float m2, float s2) {
    const float mn = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.0f : s * __expf(m - mn)) + (m2 == -INFINITY ? 0.0f : s2 * __expf(m2 - mn));
    m = mn;
}

__device__ __forceinline__ void add8(float& m, float& s, const uint4& u) {
    float f[8];
    h8_to_f(u, f);
    float mv = f[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) mv = fmaxf(mv, f[j]);
    if (mv > m) {
        s = (m == -INFINITY) ? 0.0f : s * __expf(m - mv);
        m = mv;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) s += __expf(f[j] - m);
}

__global__ void __launch_bounds__(kThreads) xent_kernel(half* dl, const half* lg, int ld, const int* __restrict__ tgt,
                                                        int N, int V, float scale, const float* __restrict__ dscale,
                                                        float* __restrict__ row_loss) {
    __shared__ float sm_m[kThreads / 32], sm_s[kThreads / 32];
    __shared__ float s_row[2];
    const float gs = scale * (dscale ? __ldg(dscale) : 1.0f);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nvec = V >> 3;                       // full 8-element vectors
    for (int row = blockIdx.x; row < N; row += gridDim.x) {
        const half* z = lg + (size_t)row * ld;
        const uint4* z4 = reinterpret_cast<const uint4*>(z);
        const int t = __ldg(tgt + row);
        const bool tvalid = t >= 0 && t < V;
        // the target logit is read before any thread can overwrite the row in place
        const float zt = (row_loss && tid == 0 && tvalid) ? __half2float(z[t]) : 0.0f;
        // ---------------- pass 1: online max / sum ----------------
        float m = -INFINITY, s = 0.0f;
        int c = tid;
        for (; c + (kUnroll - 1) * kThreads < nvec; c += kUnroll * kThreads) {
            uint4 u[kUnroll];
#pragma unroll
            for (int k = 0; k < kUnroll; ++k) u[k] = __ldcg(z4 + c + k * kThreads);
#pragma unroll
            for (int k = 0; k < kUnroll; ++k) add8(m, s, u[k]);
        }
        for (; c < nvec; c += kThreads) add8(m, s, __ldcg(z4 + c));
        for (int j = nvec * 8 + tid; j < V; j += kThreads) {
            const float f = __half2float(z[j]);
            if (f > m) { s = (m == -INFINITY) ? 0.0f : s * __expf(m - f); m = f; }
            s += __expf(f - m);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
            merge(m, s, m2, s2);
        }
        if (lane == 0) { sm_m[warp] = m; sm_s[warp] = s; }
        __syncthreads();
        if (warp == 0) {
            m = lane < kThreads / 32 ? sm_m[lane] : -INFINITY;
            s = lane < kThreads / 32 ? sm_s[lane] : 0.0f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
                merge(m, s, m2, s2);
            }
            if (lane == 0) { s_row[0] = m; s_row[1] = s; }
        }
        __syncthreads();
        const float mx = s_row[0], inv = 1.0f / s_row[1];
        if (row_loss && tid == 0) {
            float l = __int_as_float(0x7fc00000);   // NaN for an invalid target
            if (tvalid) l = -logf(__expf(zt - mx) * inv + 1e-10f);
            row_loss[row] = l;
        }
        if (dl) {
            // ---------------- pass 2: gradient (row re-read from L2) --------
            const float g = tvalid ? gs : 0.0f;
            half* d = dl + (size_t)row * ld;
            uint4* d4 = reinterpret_cast<uint4*>(d);
            for (int v = tid; v < nvec; v += kThreads) {
                float f[8];
                h8_to_f(__ldcg(z4 + v), f);
#pragma unroll
                for (int j = 0; j < 8; ++j) f[j] = (__expf(f[j] - mx) * inv - (8 * v + j == t ? 1.0f : 0.0f)) * g;
                d4[v] = f_to_h8(f);
            }
            for (int j = nvec * 8 + tid; j < V; j += kThreads)
                d[j] = __float2half_rn((__expf(__half2float(z[j]) - mx) * inv - (j == t ? 1.0f : 0.0f)) * g);
        }
        __syncthreads();   // s_row / sm_* reuse by the next row
    }
}

}  // namespace
}  // namespace rbk

using namespace rbk;

extern "C" int rbk_softmax_xent_bwd(rbk_ctx* ctx, void* dlogits, const void* logits, int ld, const int* targets,
                                    int N, int V, float scale, const float* dscale, float* row_loss, void* stream) {
    RBK_REQUIRE(ctx && logits && targets && (dlogits || row_loss), "rbk_softmax_xent_bwd: null pointer");
    RBK_REQUIRE(N > 0 && V > 0 && V <= (1 << 24) && ld >= V && ld % 8 == 0,
                "rbk_softmax_xent_bwd: need 0 < V, ld >= V, ld %% 8 == 0 (V=%d ld=%d)", V, ld);
    RBK_REQUIRE((!dlogits || aligned16(dlogits)) && aligned16(logits),
                "rbk_softmax_xent_bwd: tensors must be 16-byte aligned");
    // rows in flight (one per CTA) are kept to <= 40 MB so the second pass hits L2
    const double row_bytes = 2.0 * V;
    int per_sm = (int)(40e6 / (row_bytes * ctx->num_sms));
    per_sm = per_sm < 1 ? 1 : per_sm > 4 ? 4 : per_sm;
    int grid = ctx->num_sms * per_sm;
    if (grid > N) grid = N;
    cudaStream_t st = as_stream(stream);
    ProfScope prof(ctx, st, kCatXent,
                   (double)N * V * (dlogits ? 4.0 : 2.0) + 4.0 * N + (row_loss ? 4.0 * N : 0.0));
    xent_kernel<<<grid, kThreads, 0, st>>>((half*)dlogits, (const half*)logits, ld, targets, N, V, scale, dscale,
                                           row_loss);
    RBK_LAUNCHED("xent_kernel");
    return RBK_OK;
}
