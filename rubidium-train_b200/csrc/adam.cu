// adam.cu — the fused mixed-precision tail: overflow check, unscale, optional
// per-tensor clip, AdamW over FP32 masters, FP16 copy-out, gradient zeroing
// and the loss-scaler update, in ONE cooperative launch.
//
// Phase 1 reads every gradient once: non-finite values raise a device flag and
// (when clipping) each chunk's sum of squares is kept.  A bounded grid barrier
// separates the phases.  Phase 2 applies the update only if no rank of the
// gradients overflowed, so the skip decision is one bit for the whole model
// (the reference never skips: src/model.cu:411-425, 454-488).  The last CTA
// out updates the scaler exactly as LossScaler::update
// (src/cuda_kernels.cu:102-116) and clears the flags for the next call.
//
// AdamW is the L2-coupled form of cpuops::adamw_step / adamw_step_kernel
// (src/cpu_mat.h:280-292, backup/cuda_kernels.cu.bak:462-480):
//   g' = g / scale * clip + wd p;  m = b1 m + (1-b1) g';  v = b2 v + (1-b2) g'^2
//   p -= lr (m / (1 - b1^t)) / (sqrt(v / (1 - b2^t)) + eps)
#include <cstring>
#include <vector>

#include "common.cuh"

namespace rbk {
namespace {

constexpr int kChunk = 16384;   // elements per work item (multiple of 4)

struct Chunk {
    int64_t start;
    int32_t len;
    int32_t seg;
};

struct TailParams {
    float* p;
    float* g;
    float* m;
    float* v;
    half* p16;
    int64_t n;
    const Chunk* chunks;      // null: implicit chunks of kChunk over [0, n)
    int nchunks;
    const int* seg_begin;     // [nseg + 1] chunk index ranges per segment
    float* chunk_sumsq;       // [nchunks]
    int clip;
    float max_norm;
    float lr, b1, b2, eps, wd;
    int t;
    rbk_scaler* sc;
    int* flags;               // ctx tickets
    uint64_t wait_ns;         // grid-barrier wait limit
    int withheld_cta;         // test only: this CTA does not arrive (-1: none)
    // 3: both phases in one cooperative launch (grid barrier between them).  1 / 2: one phase
    // per launch, for the sharded optimizer: phase 1 leaves its results in xbuf ([0] = 1 if a
    // gradient was non-finite, [1 + s] = segment s's sum of squares), the caller sums xbuf
    // over the ranks, phase 2 reads the sums.
    int phases;
    float* xbuf;
    int nseg;
};

__device__ __forceinline__ void chunk_range(const TailParams& P, int c, int64_t& s, int& len, int& seg) {
    if (P.chunks) {
        const Chunk ch = P.chunks[c];
        s = ch.start;
        len = ch.len;
        seg = ch.seg;
    } else {
        s = (int64_t)c * kChunk;
        const int64_t e = s + kChunk < P.n ? s + kChunk : P.n;
        len = (int)(e - s);
        seg = 0;
    }
}

__global__ void __launch_bounds__(512, 2) adam_tail_kernel(TailParams P) {
    __shared__ float s_red[32];
    __shared__ int s_flag;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    int* overflow = P.flags + kTailOverflow;
    int* barrier = P.flags + kTailBarrier;
    int* ticket = P.flags + kTailTicket;
    int* timeout = P.flags + kTailTimeout;
    const float scale = P.sc->scale;
    const float inv_scale = 1.0f / scale;

    // ---------------- phase 1: finiteness (+ sums of squares) --------------
    if (tid == 0) s_flag = 0;
    __syncthreads();
    int bad = 0;
    for (int c = blockIdx.x; (P.phases & 1) && c < P.nchunks; c += gridDim.x) {
        int64_t s;
        int len, seg;
        chunk_range(P, c, s, len, seg);
        const float4* g4 = reinterpret_cast<const float4*>(P.g + s);
        const int nv = len >> 2;
        float ss = 0.0f;
        // four independent 16-byte loads in flight per thread (one would leave HBM idle)
        int i = tid;
        for (; i + 3 * (int)blockDim.x < nv; i += 4 * blockDim.x) {
            float4 x[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) x[u] = __ldcs(g4 + i + u * blockDim.x);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                bad |= !(isfinite(x[u].x) && isfinite(x[u].y) && isfinite(x[u].z) && isfinite(x[u].w));
                ss += x[u].x * x[u].x + x[u].y * x[u].y + x[u].z * x[u].z + x[u].w * x[u].w;
            }
        }
        for (; i < nv; i += blockDim.x) {
            const float4 x = __ldcs(g4 + i);
            bad |= !(isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w));
            ss += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
        }
        if (P.clip) {
            ss = warp_sum(ss);
            if (lane == 0) s_red[warp] = ss;
            __syncthreads();
            if (warp == 0) {
                float r = lane < nw ? s_red[lane] : 0.0f;
                r = warp_sum(r);
                if (lane == 0) P.chunk_sumsq[c] = r;
            }
            __syncthreads();
        }
    }
    if (__syncthreads_or(bad) && tid == 0) atomicOr(overflow, 1);

    if (P.phases == 1) {
        // the last CTA out folds the chunk sums into per-segment sums for the exchange
        __shared__ int s_last;
        if (tid == 0) {
            __threadfence();
            s_last = atomicAdd(ticket, 1) == (int)gridDim.x - 1;
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        if (tid == 0) P.xbuf[0] = atomicAdd(overflow, 0) ? 1.0f : 0.0f;
        for (int sg = tid; P.clip && sg < P.nseg; sg += blockDim.x) {
            float ss = 0.0f;
            for (int k = P.seg_begin[sg]; k < P.seg_begin[sg + 1]; ++k) ss += P.chunk_sumsq[k];
            P.xbuf[1 + sg] = ss;
        }
        if (tid == 0) {
            *overflow = 0;
            __threadfence();
            *ticket = 0;
        }
        return;
    }

    // ---------------- bounded grid barrier ----------------------------------
    if (P.phases == 2) {
        if (tid == 0) s_flag = P.xbuf[0] != 0.0f;
    } else if (tid == 0) {
        __threadfence();
        if ((int)blockIdx.x != P.withheld_cta) atomicAdd(barrier, 1);
        const uint64_t t0 = globaltimer_ns();
        while (atomicAdd(barrier, 0) < (int)gridDim.x) {
            if (globaltimer_ns() - t0 > P.wait_ns) { atomicOr(timeout, 1); break; }
            __nanosleep(64);
        }
        __threadfence();
        s_flag = atomicAdd(overflow, 0) | atomicAdd(timeout, 0);
    }
    __syncthreads();
    const bool skip = s_flag != 0;

    // ---------------- phase 2: update ---------------------------------------
    int t = P.t > 0 ? P.t : P.sc->applied_steps + 1;
    const float c1 = 1.0f - powf(P.b1, (float)t), c2 = 1.0f - powf(P.b2, (float)t);
    const float ic1 = 1.0f / c1, ic2 = 1.0f / c2;      // bias corrections as factors
    for (int c = blockIdx.x; c < P.nchunks; c += gridDim.x) {
        int64_t s;
        int len, seg;
        chunk_range(P, c, s, len, seg);
        float4* g4 = reinterpret_cast<float4*>(P.g + s);
        const int nv = len >> 2;
        if (!skip) {
            float f = inv_scale;
            if (P.clip) {
                float ss = 0.0f;
                if (P.phases == 2) ss = P.xbuf[1 + seg];
                else for (int k = P.seg_begin[seg]; k < P.seg_begin[seg + 1]; ++k) ss += P.chunk_sumsq[k];
                const float norm = sqrtf(ss) * inv_scale;
                if (norm > P.max_norm) f *= P.max_norm / norm;
            }
            float4* p4 = reinterpret_cast<float4*>(P.p + s);
            float4* m4 = reinterpret_cast<float4*>(P.m + s);
            float4* v4 = reinterpret_cast<float4*>(P.v + s);
            for (int i = tid; i < nv; i += blockDim.x) {
                const float4 gg = g4[i];
                float4 pp = p4[i], mm = m4[i], vv = v4[i];
                float gv[4] = {gg.x, gg.y, gg.z, gg.w}, pv[4] = {pp.x, pp.y, pp.z, pp.w};
                float mv[4] = {mm.x, mm.y, mm.z, mm.w}, vw[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float gi = gv[j] * f + P.wd * pv[j];
                    mv[j] = P.b1 * mv[j] + (1.0f - P.b1) * gi;
                    vw[j] = P.b2 * vw[j] + (1.0f - P.b2) * gi * gi;
                    const float mh = mv[j] * ic1, vh = vw[j] * ic2;
                    pv[j] -= __fdividef(P.lr * mh, sqrtf(vh) + P.eps);
                }
                p4[i] = make_float4(pv[0], pv[1], pv[2], pv[3]);
                m4[i] = make_float4(mv[0], mv[1], mv[2], mv[3]);
                v4[i] = make_float4(vw[0], vw[1], vw[2], vw[3]);
                g4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (P.p16) {
                    __half2 h[2] = {__floats2half2_rn(pv[0], pv[1]), __floats2half2_rn(pv[2], pv[3])};
                    reinterpret_cast<uint2*>(P.p16 + s)[i] = *reinterpret_cast<uint2*>(h);
                }
            }
        } else {
            for (int i = tid; i < nv; i += blockDim.x) g4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }

    // ---------------- last CTA: scaler update + flag reset -------------------
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(ticket, 1) == (int)gridDim.x - 1) {
            __threadfence();
            rbk_scaler* sc = P.sc;
            const int to = atomicAdd(timeout, 0);
            if (skip) {
                sc->unskipped = 0;
                float ns = sc->scale * 0.5f;
                sc->scale = ns < 1.0f ? 1.0f : ns;
                sc->skipped = 1;
                sc->overflow_steps += 1;
            } else {
                sc->skipped = 0;
                sc->applied_steps += 1;
                sc->unskipped += 1;
                if (sc->unskipped >= sc->interval) {
                    float ns = sc->scale * 2.0f;
                    sc->scale = ns > 65536.0f ? 65536.0f : ns;
                    sc->unskipped = 0;
                }
            }
            sc->status = to ? RBK_ERR_TIMEOUT : 0;
            *overflow = 0;
            *barrier = 0;
            *timeout = 0;
            __threadfence();
            *ticket = 0;
        }
    }
}

struct TailCache {
    std::vector<int64_t> off, len, own;
    int64_t n = -1;
    Chunk* chunks = nullptr;
    int* seg_begin = nullptr;
    float* sumsq = nullptr;
    int nchunks = 0;
    int device = -1;
};

// Cached chunk tables, keyed by the segment list and (sharded optimizer) the ranges this rank
// owns: one for the full arena, one for a shard.  Chunks are ordered by segment, each the part
// of a segment inside one owned range (the whole arena when `own` is empty), at most kChunk long.
int tail_table(rbk_ctx* ctx, const rbk_tail_args* a, const std::vector<int64_t>& own, TailCache** out) {
    static thread_local TailCache caches[2];
    TailCache& c = caches[own.empty() ? 0 : 1];
    const bool same = c.device == ctx->device && c.n == a->n && (int)c.off.size() == a->nseg &&
                      std::memcmp(c.off.data(), a->seg_off, sizeof(int64_t) * a->nseg) == 0 &&
                      std::memcmp(c.len.data(), a->seg_len, sizeof(int64_t) * a->nseg) == 0 && c.own == own;
    if (!same) {
        std::vector<Chunk> ch;
        std::vector<int> sb(a->nseg + 1);
        const std::vector<int64_t> whole = {0, a->n};
        const std::vector<int64_t>& rg = own.empty() ? whole : own;     // [begin, end) pairs, ascending
        for (int s = 0; s < a->nseg; ++s) {
            sb[s] = (int)ch.size();
            RBK_REQUIRE(a->seg_off[s] % 4 == 0 && a->seg_len[s] % 4 == 0 && a->seg_off[s] >= 0 &&
                            a->seg_off[s] + a->seg_len[s] <= a->n,
                        "rbk_adam_tail: segment %d must be 4-element aligned and inside [0, n)", s);
            for (size_t r = 0; r + 1 < rg.size(); r += 2) {
                const int64_t b = std::max(rg[r], a->seg_off[s]);
                const int64_t e = std::min(rg[r + 1], a->seg_off[s] + a->seg_len[s]);
                for (int64_t o = b; o < e; o += kChunk) {
                    const int64_t l = e - o < kChunk ? e - o : kChunk;
                    ch.push_back(Chunk{o, (int32_t)l, s});
                }
            }
        }
        sb[a->nseg] = (int)ch.size();
        if (c.chunks) cudaFree(c.chunks);
        if (c.seg_begin) cudaFree(c.seg_begin);
        if (c.sumsq) cudaFree(c.sumsq);
        c.chunks = nullptr; c.seg_begin = nullptr; c.sumsq = nullptr;
        c.n = -1;
        RBK_CUDA(cudaMalloc(&c.chunks, sizeof(Chunk) * (ch.size() + 1)));
        RBK_CUDA(cudaMalloc(&c.seg_begin, sizeof(int) * sb.size()));
        RBK_CUDA(cudaMalloc(&c.sumsq, sizeof(float) * (ch.size() + 1)));
        RBK_CUDA(cudaMemcpy(c.chunks, ch.data(), sizeof(Chunk) * ch.size(), cudaMemcpyHostToDevice));
        RBK_CUDA(cudaMemcpy(c.seg_begin, sb.data(), sizeof(int) * sb.size(), cudaMemcpyHostToDevice));
        c.off.assign(a->seg_off, a->seg_off + a->nseg);
        c.len.assign(a->seg_len, a->seg_len + a->nseg);
        c.own = own;
        c.nchunks = (int)ch.size();
        c.n = a->n;
        c.device = ctx->device;
    }
    *out = &c;
    return RBK_OK;
}

}  // namespace

// One tail launch.  own: [begin, end) pairs this rank updates (empty: the whole arena);
// phases 3 = the fused cooperative launch, 1 / 2 = one phase of the sharded optimizer with
// its exchange buffer xbuf.
int tail_launch(rbk_ctx* ctx, const rbk_tail_args* a, const std::vector<int64_t>& own, int phases, float* xbuf,
                cudaStream_t st) {
    RBK_REQUIRE(ctx && a && a->p32 && a->g && a->m && a->v && a->scaler, "rbk_adam_tail: null pointer");
    RBK_REQUIRE(a->n > 0 && a->n % 4 == 0, "rbk_adam_tail: n must be a positive multiple of 4");
    RBK_REQUIRE(aligned16(a->p32) && aligned16(a->g) && aligned16(a->m) && aligned16(a->v) &&
                    (!a->p16 || ((uintptr_t)a->p16 & 7) == 0),
                "rbk_adam_tail: masters/grads/moments need 16-byte, p16 8-byte alignment");
    const bool clip = a->max_norm > 0.0f && a->nseg > 0 && a->seg_off && a->seg_len;
    TailParams P;
    P.p = a->p32; P.g = a->g; P.m = a->m; P.v = a->v; P.p16 = (half*)a->p16; P.n = a->n;
    P.clip = clip ? 1 : 0;
    P.max_norm = a->max_norm;
    P.lr = a->lr; P.b1 = a->beta1; P.b2 = a->beta2; P.eps = a->eps; P.wd = a->weight_decay;
    P.t = a->t;
    P.sc = a->scaler;
    P.flags = ctx->tickets;
    P.wait_ns = ctx->test_tail_wait_ns ? ctx->test_tail_wait_ns : kWaitTimeoutNs;
    P.withheld_cta = ctx->test_tail_withheld_cta;
    ctx->test_tail_wait_ns = 0;                        // the test setting covers one launch
    ctx->test_tail_withheld_cta = -1;
    P.phases = phases;
    P.xbuf = xbuf;
    P.nseg = clip ? a->nseg : 1;
    int64_t whole_off = 0, whole_len = a->n;
    rbk_tail_args one = *a;
    if (!clip) {                                       // chunks of the owned ranges, one segment
        one.seg_off = &whole_off;
        one.seg_len = &whole_len;
        one.nseg = 1;
    }
    int64_t work = a->n;
    if (clip || !own.empty()) {
        TailCache* tc;
        RBK_TRY(tail_table(ctx, &one, own, &tc));
        P.chunks = tc->chunks;
        P.nchunks = tc->nchunks;
        P.seg_begin = tc->seg_begin;
        P.chunk_sumsq = tc->sumsq;
        if (!own.empty()) {
            work = 0;
            for (size_t r = 0; r + 1 < own.size(); r += 2) work += own[r + 1] - own[r];
        }
    } else {
        P.chunks = nullptr;
        P.nchunks = (int)((a->n + kChunk - 1) / kChunk);
        P.seg_begin = nullptr;
        P.chunk_sumsq = nullptr;
    }
    RBK_REQUIRE(P.nchunks > 0, "rbk_adam_tail: nothing to update");
    static thread_local int occ = 0, occ_dev = -1;
    if (occ_dev != ctx->device) {
        RBK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, adam_tail_kernel, 512, 0));
        occ_dev = ctx->device;
    }
    int grid = ctx->num_sms * (occ > 0 ? occ : 1);
    if (grid > P.nchunks) grid = P.nchunks;
    if (P.withheld_cta >= grid) P.withheld_cta = grid - 1;
    void* args[] = {&P};
    // algorithmic bytes: read g, p, m, v; write p, m, v, g (zero), p16 (phase 1: read g)
    const double per = phases == 1 ? 4.0 : phases == 2 ? (a->p16 ? 30.0 : 28.0) : (a->p16 ? 34.0 : 32.0);
    ProfScope prof(ctx, st, kCatTail, (double)work * per);
    if (phases == 3)
        RBK_CUDA(cudaLaunchCooperativeKernel((const void*)adam_tail_kernel, dim3(grid), dim3(512), args, 0, st));
    else
        RBK_CUDA(cudaLaunchKernel((const void*)adam_tail_kernel, dim3(grid), dim3(512), args, 0, st));
    count_launch();
    return RBK_OK;
}

}  // namespace rbk

using namespace rbk;

extern "C" int rbk_adam_tail(rbk_ctx* ctx, const rbk_tail_args* a, void* stream) {
    return tail_launch(ctx, a, std::vector<int64_t>(), 3, nullptr, as_stream(stream));
}
