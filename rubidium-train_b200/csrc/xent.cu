// xent.cu — fused softmax-cross-entropy forward + backward (HBM-bound).
//
// Rows that fit twice in shared memory (V up to ~56K FP16) take the ring
// kernel: one persistent CTA per SM, a producer thread bulk-copies whole rows
// into a 2-4 deep shared-memory ring, and two groups of 8 warps (alternate
// rows) make three passes over each staged row (max, sum of exp, gradient) —
// DRAM sees exactly one read and one write per logit, in place if the caller
// wishes, with the next rows already in flight.  Wider rows take the streaming kernel: pass 1 reads the row once
// with 16-byte loads and keeps an online (max, sum of exp) per thread; pass 2
// re-reads it from L2 (rows in flight are capped well below the 126 MB L2)
// and writes the gradient.  The reference instead rescans the whole row for
// every element (src/cuda_kernels.cu:533-551, O(N V^2)); cpuops does three
// passes (src/cpu_mat.h:220-236).  Per-row loss follows src/cpu_mat.h:213
// (-log(p_t + 1e-10)).
#include <cfloat>

#include "tc.cuh"

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

constexpr int kRingConsumers = 512;

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

// Ring kernel: shared memory = nbuf row buffers (rowb bytes each, V rounded up
// to 8 halves), then per-row reduction scratch red[2][2][2][32] and barriers.
// ngrp consumer groups take rows in turn: two groups of 8 warps when the ring
// holds three or more rows (each group's rows overlap the other's), one group
// of all 16 warps when only two rows fit (a 50K-logit row is 100 KB): with two
// groups there each group would wait for its own buffer's next load after every
// row, whereas one group works on a row while the other buffer loads the next.
template <int NGRP>
__global__ void __launch_bounds__(kRingConsumers + 32, 1)
    xent_ring_kernel(half* dl, const half* lg, int ld, const int* __restrict__ tgt, int N, int V, float scale,
                     const float* __restrict__ dscale, float* __restrict__ row_loss, int nbuf, int rowb, int* err) {
    using namespace tc;
    extern __shared__ __align__(128) uint8_t xs[];
    float* red = reinterpret_cast<float*>(xs + (size_t)nbuf * rowb);   // [2 groups][2 parity][2 (max, sum)][32]
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + 256);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * nbuf);
    auto full = [&](int b) { return su32(bars + b); };
    auto empty = [&](int b) { return su32(bars + nbuf + b); };
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = kRingConsumers / 32;
    if (tid == 0) {
        for (int b = 0; b < nbuf; ++b) {
            mbar_init(full(b), 1);
            mbar_init(empty(b), NW / NGRP);              // the warps of the group that took the row
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    grid_dependency_sync();
    const int nchunk = (V + 7) >> 3;                    // 16-byte chunks per row (tail masked)
    if (tid >= kRingConsumers) {
        // ------------------------------------------------------ producer ----
        if (tid == kRingConsumers) {
            int k = 0;
            for (int row = blockIdx.x; row < N; row += gridDim.x, ++k) {
                const int b = k % nbuf;
                if (!mbar_wait(empty(b), ((k / nbuf) & 1) ^ 1, abort_flag)) break;
                mbar_expect_tx(full(b), (uint32_t)(nchunk * 16));
                bulk_load(su32(xs + (size_t)b * rowb), lg + (size_t)row * ld, (uint32_t)(nchunk * 16), full(b));
            }
        }
        return;
    }
    // ---------------------------------------------------------- consumers ----
    // ngrp groups take rows in turn: each row's passes and barriers involve its group only
    const float gs = scale * (dscale ? __ldg(dscale) : 1.0f);
    constexpr float kL2e = 1.4426950408889634f;
    constexpr int GT = kRingConsumers / NGRP, GW = GT / 32;   // threads / warps per group
    const int grp = warp / GW, gtid = tid - grp * GT;
    bool ok = true;
    int k = 0, kk = 0;
    for (int row = blockIdx.x; row < N; row += gridDim.x, ++k) {
        if (k % NGRP != grp) continue;
        const int b = k % nbuf;
        const int t = __ldg(tgt + row);
        const bool tvalid = t >= 0 && t < V;
        ok = __all_sync(0xffffffffu, ok && mbar_wait(full(b), (k / nbuf) & 1, abort_flag));
        const uint32_t rb = su32(xs + (size_t)b * rowb);
        float* rr = red + (grp * 2 + (kk & 1)) * 64;
        ++kk;
        const int full8 = V >> 3;                       // chunks without a tail
        // the target logit is read before pass 2 overwrites the staged row
        const float zt = (row_loss && gtid == 0 && tvalid && ok)
                             ? __half2float(reinterpret_cast<const half*>(xs + (size_t)b * rowb)[t])
                             : 0.0f;
        // pass 1: row max
        float m = -INFINITY;
        if (ok) {
            for (int c = gtid; c < nchunk; c += GT) {
                float f[8];
                h8_to_f(lds128(rb + 16u * c), f);
                if (c < full8) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) m = fmaxf(m, f[j]);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) m = fmaxf(m, 8 * c + j < V ? f[j] : -INFINITY);
                }
            }
        }
        m = warp_max(m);
        if (lane == 0) rr[warp - grp * GW] = m;
        named_sync(1 + grp, GT);
        m = warp_max(lane < GW ? rr[lane] : -INFINITY);   // every warp folds the group's partials
        // pass 2: p = exp(z - max) (exp2 of the log2e-scaled difference), summed in FP32 and
        // written back over the staged row as FP16 (p <= 1) so pass 3 needs no second exp
        const float mb = m * kL2e;
        float sum = 0.0f;
        if (ok) {
            for (int c = gtid; c < nchunk; c += GT) {
                float f[8];
                h8_to_f(lds128(rb + 16u * c), f);
#pragma unroll
                for (int j = 0; j < 8; ++j) f[j] = ex2(fmaf(f[j], kL2e, -mb));
                if (c >= full8) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) f[j] = 8 * c + j < V ? f[j] : 0.0f;
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) sum += f[j];
                const uint4 u = f_to_h8(f);
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rb + 16u * c), "r"(u.x), "r"(u.y),
                             "r"(u.z), "r"(u.w)
                             : "memory");
            }
        }
        sum = warp_sum(sum);
        if (lane == 0) rr[32 + warp - grp * GW] = sum;
        named_sync(1 + grp, GT);                        // also orders the group's p stores before pass 3
        sum = warp_sum(lane < GW ? rr[32 + lane] : 0.0f);
        const float inv = 1.0f / sum;
        if (row_loss && gtid == 0) {
            float l = __int_as_float(0x7fc00000);       // NaN for an invalid target
            if (tvalid) l = -logf(ex2(fmaf(zt, kL2e, -mb)) * inv + 1e-10f);
            row_loss[row] = l;
        }
        // pass 3: gradient = (p / sum - onehot) * scale, 16-byte stores
        if (dl && ok) {
            const float g = tvalid ? gs : 0.0f, gi = g * inv;
            half* d = dl + (size_t)row * ld;
            for (int c = gtid; c < nchunk; c += GT) {
                float f[8];
                h8_to_f(lds128(rb + 16u * c), f);
#pragma unroll
                for (int j = 0; j < 8; ++j) f[j] *= gi;
                const int tj = t - 8 * c;               // the one chunk that holds the target
                if ((unsigned)tj < 8u) {
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (j == tj) f[j] -= g;
                }
                if (c < full8) {
                    reinterpret_cast<uint4*>(d)[c] = f_to_h8(f);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (8 * c + j < V) d[8 * c + j] = __float2half_rn(f[j]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty(b));          // this warp is done with the buffer
    }
    if (!ok && tid == 0) atomicExch(err, RBK_ERR_TIMEOUT);
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
    // ring kernel when at least two rows fit in shared memory (two 50K-logit rows do)
    const int rowb = ((V + 7) / 8) * 16;
    int nbuf = (int)((222u << 10) / (unsigned)rowb);
    nbuf = nbuf > 4 ? 4 : nbuf;
    if (nbuf >= 2) {
        const size_t smem = (size_t)nbuf * rowb + 256 * sizeof(float) + 16 * nbuf + 16;
        static int set_dev = -1;
        if (set_dev != ctx->device) {
            RBK_CUDA(cudaFuncSetAttribute(xent_ring_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448));
            RBK_CUDA(cudaFuncSetAttribute(xent_ring_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448));
            set_dev = ctx->device;
        }
        const int rgrid = N < ctx->num_sms ? N : ctx->num_sms;
        RBK_CUDA(launch_pdl(nbuf >= 3 ? xent_ring_kernel<2> : xent_ring_kernel<1>, dim3(rgrid),
                            dim3(kRingConsumers + 32), smem, st, (half*)dlogits, (const half*)logits, ld, targets, N,
                            V, scale, dscale, row_loss, nbuf, rowb, ctx->tickets + kGemmError));
        RBK_LAUNCHED("xent_ring_kernel");
        return RBK_OK;
    }
    xent_kernel<<<grid, kThreads, 0, st>>>((half*)dlogits, (const half*)logits, ld, targets, N, V, scale, dscale,
                                           row_loss);
    RBK_LAUNCHED("xent_kernel");
    return RBK_OK;
}
