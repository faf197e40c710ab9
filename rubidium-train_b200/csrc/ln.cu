// ln.cu — LayerNorm forward and backward over FP16 rows (HBM-bound).
//
// Forward: one warp per row, the row held in registers (16-byte vectors), two
// passes over registers for mean and biased variance, as
// layer_norm_fp16_fwd_kernel / cpuops::layer_norm (reference
// src/cuda_kernels.cu:183-225, src/cpu_mat.h:98-123).
//
// Backward: a "team" of D/8 threads covers one row, each thread owning 8
// adjacent columns, and several teams share a CTA.  A thread keeps its
// columns' dgamma / dbeta (/ dbias) partial sums in registers for every row
// its team visits, instead of the reference's per-element half atomics
// (src/cuda_kernels.cu:279-282).  One persistent CTA per SM streams blocks of
// consecutive rows of dy, x (and the residual gradient) into a shared-memory
// ring with bulk copies issued by one producer thread, so 100+ KB per SM are
// in flight while the teams work; each team reduces its two row sums through
// shared memory behind its own named barrier.  At the end the teams of a CTA
// fold their partials in shared memory, and one small column-parallel launch
// sums the per-CTA partials in a fixed order, so results are bitwise
// reproducible.
#include "tc.cuh"

namespace rbk {
namespace {

// One warp per row, NV 16-byte vectors per lane.  Each warp walks its rows with the next
// row's vectors already in flight while it works on the current one.  For D <= 1024
// (NV <= 4) the current row is held as FP32 and gamma / beta stay in registers; for
// 1024 < D <= 2048 the row stays FP16 and is converted again in each of the three passes
// (sum, centred sum of squares, output), gamma / beta come from L1, so two rows fit the
// registers of two CTAs per SM; wider rows load each row when they reach it.
template <int NV>
__global__ void __launch_bounds__(256) ln_fwd_kernel(half* __restrict__ y, float* __restrict__ mean,
                                                     float* __restrict__ rstd, const half* __restrict__ x,
                                                     const half* __restrict__ g, const half* __restrict__ b, int N,
                                                     int D, float eps) {
    grid_dependency_sync();
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    const int nvec = D >> 3;
    const float invD = 1.0f / (float)D;
    const int stride = gridDim.x * warps;
    constexpr bool kPrefetch = NV <= 4;
    if constexpr (NV > 4 && NV <= 8) {
        uint4 cur[NV], nxt[NV];
        int row = blockIdx.x * warps + (threadIdx.x >> 5);
        auto load = [&](uint4* dst, int r) {
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int c = lane + 32 * i;
                dst[i] = (r < N && c < nvec) ? __ldg(reinterpret_cast<const uint4*>(x + (size_t)r * D) + c)
                                             : make_uint4(0, 0, 0, 0);
            }
        };
        load(nxt, row);
        for (; row < N; row += stride) {
#pragma unroll
            for (int i = 0; i < NV; ++i) cur[i] = nxt[i];
            load(nxt, row + stride);                         // next row in flight during this one
            float s = 0.0f;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                float v[8];
                h8_to_f(cur[i], v);
#pragma unroll
                for (int j = 0; j < 8; ++j) s += v[j];
            }
            const float m = warp_sum(s) * invD;
            float q = 0.0f;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                if (lane + 32 * i < nvec) {
                    float v[8];
                    h8_to_f(cur[i], v);
#pragma unroll
                    for (int j = 0; j < 8; ++j) { const float d = v[j] - m; q += d * d; }
                }
            }
            const float r = 1.0f / sqrtf(warp_sum(q) * invD + eps);
            uint4* yr = reinterpret_cast<uint4*>(y + (size_t)row * D);
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const int c = lane + 32 * i;
                if (c < nvec) {
                    float v[8], gf[8], bf[8], o[8];
                    h8_to_f(cur[i], v);
                    h8_to_f(__ldg(reinterpret_cast<const uint4*>(g) + c), gf);
                    h8_to_f(__ldg(reinterpret_cast<const uint4*>(b) + c), bf);
#pragma unroll
                    for (int j = 0; j < 8; ++j) o[j] = gf[j] * (v[j] - m) * r + bf[j];
                    yr[c] = f_to_h8(o);
                }
            }
            if (lane == 0) { mean[row] = m; rstd[row] = r; }
        }
        return;
    }
    uint4 gr[kPrefetch ? NV : 1], br[kPrefetch ? NV : 1], nx[NV];
    if constexpr (kPrefetch) {
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int c = lane + 32 * i;
            gr[i] = c < nvec ? __ldg(reinterpret_cast<const uint4*>(g) + c) : make_uint4(0, 0, 0, 0);
            br[i] = c < nvec ? __ldg(reinterpret_cast<const uint4*>(b) + c) : make_uint4(0, 0, 0, 0);
        }
    }
    int row = blockIdx.x * warps + (threadIdx.x >> 5);
    auto load_row = [&](int r) {
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int c = lane + 32 * i;
            nx[i] = (r < N && c < nvec) ? __ldg(reinterpret_cast<const uint4*>(x + (size_t)r * D) + c)
                                        : make_uint4(0, 0, 0, 0);
        }
    };
    if constexpr (kPrefetch) load_row(row);
    for (; row < N; row += stride) {
        if constexpr (!kPrefetch) load_row(row);
        float v[NV][8];
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            h8_to_f(nx[i], v[i]);
#pragma unroll
            for (int j = 0; j < 8; ++j) s += v[i][j];
        }
        if constexpr (kPrefetch) load_row(row + stride);   // next row in flight during the reductions
        const float m = warp_sum(s) * invD;
        float q = 0.0f;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int c = lane + 32 * i;
            if (c < nvec) {
#pragma unroll
                for (int j = 0; j < 8; ++j) { const float d = v[i][j] - m; q += d * d; }
            }
        }
        const float r = 1.0f / sqrtf(warp_sum(q) * invD + eps);
        uint4* yr = reinterpret_cast<uint4*>(y + (size_t)row * D);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int c = lane + 32 * i;
            if (c < nvec) {
                float gf[8], bf[8], o[8];
                if constexpr (kPrefetch) {
                    h8_to_f(gr[i], gf);
                    h8_to_f(br[i], bf);
                } else {
                    h8_to_f(__ldg(reinterpret_cast<const uint4*>(g) + c), gf);
                    h8_to_f(__ldg(reinterpret_cast<const uint4*>(b) + c), bf);
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) o[j] = gf[j] * (v[i][j] - m) * r + bf[j];
                yr[c] = f_to_h8(o);
            }
        }
        if (lane == 0) { mean[row] = m; rstd[row] = r; }
    }
}

constexpr int kLnRows = 4;       // rows per team iteration in the backward (the butterfly assumes 4)
constexpr int kLnMaxTeams = 8;

// Dynamic shared memory: red[2][teams][2R][warps per team] then part[teams][3][D].
// part (global) layout: [gridDim.x][3][D]  (dgamma | dbeta | dbias partials)
template <bool kRefFormula, bool kRes, bool kBias>
__global__ void __launch_bounds__(512) ln_bwd_kernel(half* __restrict__ dx, float* __restrict__ part,
                                                      const half* __restrict__ dy, const half* __restrict__ dres,
                                                      const half* __restrict__ x, const half* __restrict__ g,
                                                      const float* __restrict__ mean, const float* __restrict__ rstd,
                                                      int N, int D, int teams) {
    constexpr int R = kLnRows;
    extern __shared__ float lsm[];
    const int tpt = blockDim.x / teams;                 // threads per team
    const int wpt = tpt >> 5;                           // warps per team
    const int tid = threadIdx.x, team = tid / tpt, ttid = tid - team * tpt;
    const int lane = tid & 31, twarp = ttid >> 5;
    float* red = lsm;                                   // [2][teams][2R][wpt]
    float* tpart = lsm + 2 * teams * 2 * R * wpt;       // [teams][3][D]
    const int nvec = D >> 3;
    const bool own = ttid < nvec;                       // columns [8 ttid, 8 ttid + 8)
    const float invD = 1.0f / (float)D;
    float gam[8], pg[8], pb[8], pd[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) { pg[j] = 0.0f; pb[j] = 0.0f; pd[j] = 0.0f; gam[j] = 0.0f; }
    if (own) h8_to_f(__ldg(reinterpret_cast<const uint4*>(g) + ttid), gam);

    const int ngroups = (N + R - 1) / R;
    const int stride = gridDim.x * teams;
    const int iters = (ngroups + stride - 1) / stride;
    for (int it = 0; it < iters; ++it) {
        const int buf = it & 1;
        const int grp = it * stride + blockIdx.x * teams + team;
        const int row0 = grp * R;
        uint4 dyv[R], xv[R];
        float mr[R], rr[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int row = row0 + r;
            const bool rowok = grp < ngroups && row < N;
            const bool ok = own && rowok;
            dyv[r] = ok ? __ldg(reinterpret_cast<const uint4*>(dy + (size_t)row * D) + ttid) : make_uint4(0, 0, 0, 0);
            xv[r] = ok ? __ldg(reinterpret_cast<const uint4*>(x + (size_t)row * D) + ttid) : make_uint4(0, 0, 0, 0);
            mr[r] = rowok ? __ldg(mean + row) : 0.0f;
            rr[r] = rowok ? __ldg(rstd + row) : 0.0f;
        }
        // Row sums: ts1 = sum dy*g, ts2 = sum dy*g*(x - mean).
        float ts[2 * R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            float d[8], xx[8];
            h8_to_f(dyv[r], d);
            h8_to_f(xv[r], xx);
            float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float dg = d[j] * gam[j];
                s1 += dg;
                s2 += dg * (xx[j] - mr[r]);
            }
            ts[2 * r] = warp_sum(s1);
            ts[2 * r + 1] = warp_sum(s2);
        }
        float* rb = red + ((size_t)buf * teams + team) * 2 * R * wpt;
        if (lane == 0) {
#pragma unroll
            for (int k = 0; k < 2 * R; ++k) rb[k * wpt + twarp] = ts[k];
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 2 * R; ++k) {
            float s = 0.0f;
            for (int w = 0; w < wpt; ++w) s += rb[k * wpt + w];
            ts[k] = s;
        }
        // (the other buffer is written next iteration; this barrier orders the
        //  reads of `buf` before the iteration after next overwrites it)
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int row = row0 + r;
            if (own && grp < ngroups && row < N) {
                float d[8], xx[8], o[8];
                h8_to_f(dyv[r], d);
                h8_to_f(xv[r], xx);
                float rs[8];
                if (kRes) h8_to_f(__ldg(reinterpret_cast<const uint4*>(dres + (size_t)row * D) + ttid), rs);
                const float inv = rr[r];
                const float c2 = kRefFormula ? inv : inv * inv;
                const float t1 = ts[2 * r], t2 = ts[2 * r + 1];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float xm = xx[j] - mr[r];
                    float v = inv * (d[j] * gam[j] - (t1 + xm * c2 * t2) * invD);
                    if (kRes) v += rs[j];
                    o[j] = v;
                    pg[j] += d[j] * xm * inv;
                    pb[j] += d[j];
                    if (kBias) pd[j] += v;
                }
                reinterpret_cast<uint4*>(dx + (size_t)row * D)[ttid] = f_to_h8(o);
            }
        }
    }
    // fold the teams' partials in shared memory, then one CTA partial to global
    if (own) {
        float* tp = tpart + (size_t)team * 3 * D + 8 * ttid;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            tp[j] = pg[j];
            tp[D + j] = pb[j];
            tp[2 * D + j] = pd[j];
        }
    }
    __syncthreads();
    for (int i = tid; i < 3 * D; i += blockDim.x) {
        float s = 0.0f;
        for (int t = 0; t < teams; ++t) s += tpart[(size_t)t * 3 * D + i];
        part[(size_t)blockIdx.x * 3 * D + i] = s;
    }
}

// out_w[c] += sum_b part[b][w][c] for w in {dgamma, dbeta, dbias}: 32 columns per
// CTA (one per lane), the 32 warps split the partial rows (all their loads in
// flight at once), fixed summation order.
__global__ void __launch_bounds__(1024) ln_bwd_reduce_kernel(float* __restrict__ dg, float* __restrict__ db,
                                                             float* __restrict__ dbias,
                                                             const float* __restrict__ part, int nblk, int D) {
    // launched as a programmatic dependent of the main pass: wait for its partials
    grid_dependency_sync();
    __shared__ float s[32][33];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    const int which = blockIdx.y;
    float* out = which == 0 ? dg : which == 1 ? db : dbias;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (c < D) {
        int b = warp;
        for (; b + 96 < nblk; b += 128) {
#pragma unroll
            for (int u = 0; u < 4; ++u) acc[u] += __ldg(part + (size_t)(b + 32 * u) * 3 * D + (size_t)which * D + c);
        }
        for (; b < nblk; b += 32) acc[0] += __ldg(part + (size_t)b * 3 * D + (size_t)which * D + c);
    }
    s[warp][lane] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    __syncthreads();
    if (warp == 0 && c < D && out) {
        float t = 0.0f;
#pragma unroll 8
        for (int w = 0; w < 32; ++w) t += s[w][lane];
        out[c] += t;
    }
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ float4 lds128f(uint32_t addr) {
    const uint4 u = lds128(addr);
    return make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w));
}

// ---------------------------------------------------------------------------
// Backward with a bulk-copy ring.  Shared memory: stages x [dy | x | dres] row
// blocks (kLnRows consecutive rows of D halves each, one bulk copy per tensor;
// stage k belongs to team k % teams, so teams release their stages
// independently), the teams' row-sum exchange red[teams][2][2 kLnRows][warps
// per team], barriers; at the end the ring is reused for the teams' column
// partials tpart[teams][3][D].
// part (global) layout: [gridDim.x][3][D]  (dgamma | dbeta | dbias partials)
template <bool kRefFormula, bool kRes, bool kBias>
__global__ void __launch_bounds__(544, 1)
    ln_bwd_ring_kernel(half* __restrict__ dx, float* __restrict__ part, const half* __restrict__ dy,
                       const half* __restrict__ dres, const half* __restrict__ x, const half* __restrict__ g,
                       const float* __restrict__ mean, const float* __restrict__ rstd, int N, int D, int teams,
                       int tpt, int stages, int* err) {
    using namespace tc;
    constexpr int R = kLnRows;
    static_assert(R == 4, "the row-sum butterfly below reduces 2 * 4 sums");
    constexpr int NT = kRes ? 3 : 2;
    extern __shared__ __align__(128) uint8_t lsm_raw[];
    const int RS = R;                                   // rows per stage: one team's rows
    const size_t row_bytes = (size_t)D * 2;
    const size_t stage_bytes = (size_t)RS * row_bytes * NT;
    const int wpt = tpt >> 5;
    float* red = reinterpret_cast<float*>(lsm_raw + stages * stage_bytes);    // [teams][2][2R][wpt]
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + (size_t)teams * 2 * 2 * R * wpt);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * stages);
    auto full = [&](int s) { return su32(bars + s); };
    auto empty = [&](int s) { return su32(bars + stages + s); };
    const int consumers = teams * tpt;                  // consumer threads; one producer warp follows
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), tpt >> 5);              // the warps of the team that owns the stage
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    grid_dependency_wait();                             // dependents are released at the end
    const int nstage = (N + RS - 1) / RS;

    if (tid >= consumers) {
        // ------------------------------------------------------ producer ----
        if (tid == consumers) {
            int k = 0;
            for (int gs = blockIdx.x; gs < nstage; gs += gridDim.x, ++k) {
                const int s = k % stages;
                if (!mbar_wait(empty(s), ((k / stages) & 1) ^ 1, abort_flag)) break;
                const int rows = min(RS, N - gs * RS);
                mbar_expect_tx(full(s), (uint32_t)(rows * row_bytes * NT));
                const uint32_t dst = su32(lsm_raw + s * stage_bytes);
                const size_t off = (size_t)gs * RS * D;
                const uint32_t bytes = (uint32_t)(rows * row_bytes);   // consecutive rows: one copy per tensor
                bulk_load(dst, dy + off, bytes, full(s));
                bulk_load(dst + (uint32_t)(RS * row_bytes), x + off, bytes, full(s));
                if (kRes) bulk_load(dst + (uint32_t)(2 * RS * row_bytes), dres + off, bytes, full(s));
            }
        }
    } else {
        // ------------------------------------------------------ consumers ----
        const int team = tid / tpt, ttid = tid - team * tpt, twarp = ttid >> 5;
        const int nvec = D >> 3;
        const bool own = ttid < nvec;                   // columns [8 ttid, 8 ttid + 8)
        const float invD = 1.0f / (float)D;
        // packed FP32 pairs (sm_100 f32x2 arithmetic) over the thread's 8 columns
        uint64_t gam[4], pg[4], pb[4], pd[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) { pg[j] = 0; pb[j] = 0; pd[j] = 0; gam[j] = 0; }
        if (own) h8_to_p(__ldg(reinterpret_cast<const uint4*>(g) + ttid), gam);
        bool ok = true;
        const uint32_t ring = su32(lsm_raw);
        // this team's row statistics are loaded one stage ahead, so their latency hides behind a stage
        float nmr[R], nrr[R];
        {
            const int row0 = (blockIdx.x + team * gridDim.x) * RS;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                nmr[r] = row0 + r < N ? __ldg(mean + row0 + r) : 0.0f;
                nrr[r] = row0 + r < N ? __ldg(rstd + row0 + r) : 0.0f;
            }
        }
        int it = 0;
        for (int k = team; blockIdx.x + k * gridDim.x < nstage; k += teams, ++it) {
            const int gs = blockIdx.x + k * gridDim.x;
            const int s = k % stages;
            const int row0 = gs * RS;
            float mr[R], rr[R];
            const int nrow0 = (blockIdx.x + (k + teams) * gridDim.x) * RS;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                mr[r] = nmr[r];
                rr[r] = nrr[r];
                nmr[r] = nrow0 + r < N ? __ldg(mean + nrow0 + r) : 0.0f;
                nrr[r] = nrow0 + r < N ? __ldg(rstd + nrow0 + r) : 0.0f;
            }
            ok = __all_sync(0xffffffffu, ok && mbar_wait(full(s), (k / stages) & 1, abort_flag));
            const uint32_t sb = ring + (uint32_t)(s * stage_bytes);
            // pass 1 over the staged rows: ts1 = sum dy*g, ts2 = sum dy*g*(x - mean)
            float v8[2 * R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int lr = r;                       // row inside the stage
                float s1 = 0.0f, s2 = 0.0f;
                if (ok && own && row0 + r < N) {
                    uint64_t d[4], xx[4];
                    h8_to_p(lds128(sb + (uint32_t)(lr * row_bytes + 16 * ttid)), d);
                    h8_to_p(lds128(sb + (uint32_t)((RS + lr) * row_bytes + 16 * ttid)), xx);
                    const uint64_t m2 = pk2(mr[r], mr[r]);
                    uint64_t a1 = 0, a2 = 0;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint64_t dg = pmul2(d[j], gam[j]);
                        a1 = padd2(a1, dg);
                        a2 = pfma2(dg, psub2(xx[j], m2), a2);
                    }
                    s1 = lo2(a1) + hi2(a1);
                    s2 = lo2(a2) + hi2(a2);
                }
                v8[2 * r] = s1;
                v8[2 * r + 1] = s2;
            }
            // warp totals of the 8 sums with one transposed butterfly (9 shuffles): lane l ends with
            // the total of sum index (l >> 2) & 7
            float tot;
            {
                const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
                float a4[4], a2[2];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float keep = b4 ? v8[i + 4] : v8[i], send = b4 ? v8[i] : v8[i + 4];
                    a4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
                }
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const float keep = b3 ? a4[i + 2] : a4[i], send = b3 ? a4[i] : a4[i + 2];
                    a2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
                }
                tot = (b2 ? a2[1] : a2[0]) + __shfl_xor_sync(0xffffffffu, b2 ? a2[0] : a2[1], 4);
                tot += __shfl_xor_sync(0xffffffffu, tot, 2);
                tot += __shfl_xor_sync(0xffffffffu, tot, 1);
            }
            float* rb = red + ((size_t)team * 2 + (it & 1)) * 2 * R * wpt;
            if ((lane & 3) == 0) rb[((lane >> 2) & 7) * wpt + twarp] = tot;
            named_sync(1 + team, tpt);                  // this team's warps only
            // lane q < 8 adds the team's warps for sum q; shuffles hand every lane all 8 totals
            float mine = 0.0f;
            if (lane < 2 * R)
                for (int w = 0; w < wpt; ++w) mine += rb[lane * wpt + w];
            float ts[2 * R];
#pragma unroll
            for (int q = 0; q < 2 * R; ++q) ts[q] = __shfl_sync(0xffffffffu, mine, q);
            // pass 2: dx = A * dy*g + B * xhat + C per row, column partials
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const int lr = r;
                const int row = row0 + r;
                if (ok && own && row < N) {
                    uint64_t d[4], xx[4], o[4], rs[4];
                    h8_to_p(lds128(sb + (uint32_t)(lr * row_bytes + 16 * ttid)), d);
                    h8_to_p(lds128(sb + (uint32_t)((RS + lr) * row_bytes + 16 * ttid)), xx);
                    if (kRes) h8_to_p(lds128(sb + (uint32_t)((2 * RS + lr) * row_bytes + 16 * ttid)), rs);
                    const float inv = rr[r], m = mr[r];
                    const float t1 = ts[2 * r], t2 = ts[2 * r + 1];
                    // exact: dx = inv * (dy g - (t1 + (x - m) * inv^2 * t2) / D); the reference formula
                    // has inv instead of inv^2 (one rstd factor short).  Per row constants:
                    // dx = (inv g) dy + Bx x + C
                    const float Bx = -inv * (kRefFormula ? inv : inv * inv) * t2 * invD;
                    const float C = -inv * t1 * invD - Bx * m;
                    const uint64_t inv2 = pk2(inv, inv), m2 = pk2(m, m), bx2 = pk2(Bx, Bx), c2 = pk2(C, C);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        uint64_t v = pfma2(pmul2(inv2, gam[j]), d[j], pfma2(bx2, xx[j], c2));
                        if (kRes) v = padd2(v, rs[j]);
                        o[j] = v;
                        pg[j] = pfma2(d[j], pmul2(psub2(xx[j], m2), inv2), pg[j]);
                        pb[j] = padd2(pb[j], d[j]);
                        if (kBias) pd[j] = padd2(pd[j], v);
                    }
                    reinterpret_cast<uint4*>(dx + (size_t)row * D)[ttid] = p_to_h8(o);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty(s));      // this warp is done with the stage
        }
        if (!ok && tid == 0) atomicExch(err, RBK_ERR_TIMEOUT);
        // park the partials until the ring is free (all copies were consumed)
        __syncthreads();
        float* tpart = reinterpret_cast<float*>(lsm_raw);   // [teams][3][D]
        if (own) {
            float* tp = tpart + (size_t)team * 3 * D + 8 * ttid;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                tp[2 * j] = lo2(pg[j]);
                tp[2 * j + 1] = hi2(pg[j]);
                tp[D + 2 * j] = lo2(pb[j]);
                tp[D + 2 * j + 1] = hi2(pb[j]);
                tp[2 * D + 2 * j] = lo2(pd[j]);
                tp[2 * D + 2 * j + 1] = hi2(pd[j]);
            }
        }
    }
    if (tid >= consumers) __syncthreads();              // matches the consumers' barrier above
    __syncthreads();
    const float* tpart = reinterpret_cast<const float*>(lsm_raw);
    for (int i = tid; i < 3 * D; i += blockDim.x) {
        float v = 0.0f;
        for (int t = 0; t < teams; ++t) v += tpart[(size_t)t * 3 * D + i];
        part[(size_t)blockIdx.x * 3 * D + i] = v;
    }
    // the column reduce may start launching (it waits for this grid's memory before reading)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// The ring backward specialised for D = 2048 (every column owned: D / 8 threads per
// team, a multiple of 32) with mixed-precision arithmetic, about half the instructions per
// element of the generic ring kernel, which is issue-bound:
//   - row sums t1 = sum dy g (exact products: fma.rn.f32.f16) and sum (dy g) x with FP32
//     accumulation, t2 = sum (dy g)(x - m) = that - m t1 per row (the (dy g) products rounded to
//     FP16 first; t1 and t2 enter dx only through their row means);
//   - dx = inv (dy g) - (inv^2 t2 / D) xhat - inv t1 / D in packed FP16 (the output is FP16; every
//     term is within a small factor of the output's magnitude), xhat = (x - m_hi - m_lo) inv with
//     the row mean split into two FP16 parts, so x - m keeps full precision for any mean;
//   - column sums dgamma += dy xhat and dbeta += dy in FP32 from FP32 dy and xhat (the same
//     arithmetic as the generic kernel, so the weight gradients agree with it to FP32 rounding);
//     dbias += dx accumulates the FP16 dx in FP32 (add.rn.f32.f16).
// Same ring, teams, barriers, butterfly and outputs as ln_bwd_ring_kernel.
__device__ __forceinline__ void mfma2(float& c0, float& c1, uint32_t a, uint32_t b) {
    asm("{.reg .f16 al, ah, bl, bh;\n\t"
        "mov.b32 {al, ah}, %2;\n\t"
        "mov.b32 {bl, bh}, %3;\n\t"
        "fma.rn.f32.f16 %0, al, bl, %0;\n\t"
        "fma.rn.f32.f16 %1, ah, bh, %1;}"
        : "+f"(c0), "+f"(c1)
        : "r"(a), "r"(b));
}
__device__ __forceinline__ void madd2(float& c0, float& c1, uint32_t a) {
    asm("{.reg .f16 al, ah;\n\t"
        "mov.b32 {al, ah}, %2;\n\t"
        "add.rn.f32.f16 %0, al, %0;\n\t"
        "add.rn.f32.f16 %1, ah, %1;}"
        : "+f"(c0), "+f"(c1)
        : "r"(a));
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

template <int D, bool kRefFormula, bool kRes, bool kBias>
__global__ void __launch_bounds__(D / 8 * (512 / (D / 8) > kLnMaxTeams ? kLnMaxTeams : 512 / (D / 8)) + 32, 1)
    ln_bwd_mx_kernel(half* __restrict__ dx, float* __restrict__ part, const half* __restrict__ dy,
                     const half* __restrict__ dres, const half* __restrict__ x, const half* __restrict__ g,
                     const float* __restrict__ mean, const float* __restrict__ rstd, int N, int stages, int* err) {
    using namespace tc;
    constexpr int R = kLnRows;
    static_assert(R == 4, "the row-sum butterfly below reduces 2 * 4 sums");
    constexpr int TPT = D / 8;                          // threads per team, one per 8 columns
    static_assert(TPT % 32 == 0, "whole warps per team");
    constexpr int TEAMS = 512 / TPT > kLnMaxTeams ? kLnMaxTeams : 512 / TPT;
    constexpr int WPT = TPT / 32;
    constexpr int NT = kRes ? 3 : 2;
    constexpr uint32_t ROW_BYTES = D * 2;
    constexpr uint32_t STAGE_BYTES = R * ROW_BYTES * NT;
    constexpr float kInvD = 1.0f / (float)D;
    extern __shared__ __align__(128) uint8_t lsm_raw[];
    float* red = reinterpret_cast<float*>(lsm_raw + (size_t)stages * STAGE_BYTES);   // [TEAMS][2][2R][WPT]
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + TEAMS * 2 * 2 * R * WPT);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * stages);
    auto full = [&](int s) { return su32(bars + s); };
    auto empty = [&](int s) { return su32(bars + stages + s); };
    constexpr int CONSUMERS = TEAMS * TPT;
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), WPT);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    grid_dependency_wait();
    const int nstage = (N + R - 1) / R;

    if (tid >= CONSUMERS) {
        if (tid == CONSUMERS) {                         // producer: one bulk copy per tensor per stage
            int k = 0;
            for (int gs = blockIdx.x; gs < nstage; gs += gridDim.x, ++k) {
                const int s = k % stages;
                if (!mbar_wait(empty(s), ((k / stages) & 1) ^ 1, abort_flag)) break;
                const int rows = min(R, N - gs * R);
                mbar_expect_tx(full(s), (uint32_t)rows * ROW_BYTES * NT);
                const uint32_t dst = su32(lsm_raw + (size_t)s * STAGE_BYTES);
                const size_t off = (size_t)gs * R * D;
                const uint32_t bytes = (uint32_t)rows * ROW_BYTES;
                bulk_load(dst, dy + off, bytes, full(s));
                bulk_load(dst + R * ROW_BYTES, x + off, bytes, full(s));
                if (kRes) bulk_load(dst + 2 * R * ROW_BYTES, dres + off, bytes, full(s));
            }
        }
    } else {
        const int team = tid / TPT, ttid = tid - team * TPT, twarp = ttid >> 5;
        uint32_t gam[4];                                // gamma of the thread's 8 columns, FP16 pairs
        {
            const uint4 gv = __ldg(reinterpret_cast<const uint4*>(g) + ttid);
            gam[0] = gv.x; gam[1] = gv.y; gam[2] = gv.z; gam[3] = gv.w;
        }
        uint64_t pg[4], pb[4];                          // FP32 pairs: dgamma, dbeta
        float pd[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) { pg[j] = 0; pb[j] = 0; }
#pragma unroll
        for (int j = 0; j < 8; ++j) pd[j] = 0.f;
        bool ok = true;
        const uint32_t ring = su32(lsm_raw);
        float nmr[R], nrr[R];
        {
            const int row0 = (blockIdx.x + team * gridDim.x) * R;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                nmr[r] = row0 + r < N ? __ldg(mean + row0 + r) : 0.0f;
                nrr[r] = row0 + r < N ? __ldg(rstd + row0 + r) : 0.0f;
            }
        }
        int it = 0;
        for (int k = team; blockIdx.x + k * gridDim.x < nstage; k += TEAMS, ++it) {
            const int gs = blockIdx.x + k * gridDim.x;
            const int s = k % stages;
            const int row0 = gs * R;
            const int nrows = min(R, N - row0);
            float mr[R], rr[R];
            const int nrow0 = (blockIdx.x + (k + TEAMS) * gridDim.x) * R;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                mr[r] = nmr[r];
                rr[r] = nrr[r];
                nmr[r] = nrow0 + r < N ? __ldg(mean + nrow0 + r) : 0.0f;
                nrr[r] = nrow0 + r < N ? __ldg(rstd + nrow0 + r) : 0.0f;
            }
            ok = __all_sync(0xffffffffu, ok && mbar_wait(full(s), (k / stages) & 1, abort_flag));
            const uint32_t sb = ring + (uint32_t)s * STAGE_BYTES + 16u * ttid;
            // pass 1: per row, t1 = sum dy g and sum (dy g) x over the thread's 8 columns
            float v8[2 * R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                float s1a = 0.f, s1b = 0.f, s2a = 0.f, s2b = 0.f;
                if (ok && r < nrows) {
                    const uint4 d = lds128(sb + r * ROW_BYTES);
                    const uint4 xv = lds128(sb + (R + r) * ROW_BYTES);
                    const uint32_t dd[4] = {d.x, d.y, d.z, d.w}, xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        mfma2(s1a, s1b, dd[j], gam[j]);
                        mfma2(s2a, s2b, h2u(__hmul2(u2h(dd[j]), u2h(gam[j]))), xx[j]);
                    }
                }
                v8[2 * r] = s1a + s1b;
                v8[2 * r + 1] = s2a + s2b;
            }
            float tot;
            {
                const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
                float a4[4], a2[2];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float keep = b4 ? v8[i + 4] : v8[i], send = b4 ? v8[i] : v8[i + 4];
                    a4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
                }
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const float keep = b3 ? a4[i + 2] : a4[i], send = b3 ? a4[i] : a4[i + 2];
                    a2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
                }
                tot = (b2 ? a2[1] : a2[0]) + __shfl_xor_sync(0xffffffffu, b2 ? a2[0] : a2[1], 4);
                tot += __shfl_xor_sync(0xffffffffu, tot, 2);
                tot += __shfl_xor_sync(0xffffffffu, tot, 1);
            }
            float* rb = red + ((size_t)team * 2 + (it & 1)) * 2 * R * WPT;
            if ((lane & 3) == 0) rb[((lane >> 2) & 7) * WPT + twarp] = tot;
            named_sync(1 + team, TPT);
            float mine = 0.0f;
            if (lane < 2 * R) {
#pragma unroll
                for (int w = 0; w < WPT; ++w) mine += rb[lane * WPT + w];
            }
            float ts[2 * R];
#pragma unroll
            for (int q = 0; q < 2 * R; ++q) ts[q] = __shfl_sync(0xffffffffu, mine, q);
            // pass 2
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (ok && r < nrows) {
                    const float inv = rr[r], m = mr[r];
                    const float t1 = ts[2 * r], t2 = ts[2 * r + 1] - m * t1;   // sum (dy g)(x - m)
                    // dx = inv (dy g) + bh xhat + c,  xhat = (x - m) inv
                    const float bh = -(kRefFormula ? inv : inv * inv) * t2 * kInvD;
                    const float c = -inv * t1 * kInvD;
                    const __half mhi = __float2half_rn(m);
                    const __half mlo = __float2half_rn(m - __half2float(mhi));
                    const __half2 mhi2 = __halves2half2(mhi, mhi), mlo2 = __halves2half2(mlo, mlo);
                    const __half2 inv2 = __float2half2_rn(inv), bh2 = __float2half2_rn(bh), c2 = __float2half2_rn(c);
                    const uint64_t iv2 = pk2(inv, inv), nmi2 = pk2(-m * inv, -m * inv);
                    const uint4 d = lds128(sb + r * ROW_BYTES);
                    const uint4 xv = lds128(sb + (R + r) * ROW_BYTES);
                    uint4 rv = make_uint4(0u, 0u, 0u, 0u);
                    if (kRes) rv = lds128(sb + (2 * R + r) * ROW_BYTES);
                    const uint32_t dd[4] = {d.x, d.y, d.z, d.w}, xx[4] = {xv.x, xv.y, xv.z, xv.w};
                    const uint32_t rs[4] = {rv.x, rv.y, rv.z, rv.w};
                    uint64_t df[4], xf[4];
                    h8_to_p(d, df);
                    h8_to_p(xv, xf);
                    uint32_t o[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const __half2 xh = __hmul2(__hsub2(__hsub2(u2h(xx[j]), mhi2), mlo2), inv2);
                        const __half2 dg = __hmul2(u2h(dd[j]), u2h(gam[j]));
                        __half2 v = __hfma2(inv2, dg, __hfma2(bh2, xh, c2));
                        if (kRes) v = __hadd2(v, u2h(rs[j]));
                        o[j] = h2u(v);
                        pg[j] = pfma2(df[j], pfma2(xf[j], iv2, nmi2), pg[j]);   // dy (x inv - m inv)
                        pb[j] = padd2(pb[j], df[j]);
                        if (kBias) madd2(pd[2 * j], pd[2 * j + 1], o[j]);
                    }
                    reinterpret_cast<uint4*>(dx + (size_t)(row0 + r) * D)[ttid] = make_uint4(o[0], o[1], o[2], o[3]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty(s));
        }
        if (!ok && tid == 0) atomicExch(err, RBK_ERR_TIMEOUT);
        __syncthreads();
        float* tpart = reinterpret_cast<float*>(lsm_raw);   // [TEAMS][3][D]
        float* tp = tpart + (size_t)team * 3 * D + 8 * ttid;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            tp[2 * j] = lo2(pg[j]);
            tp[2 * j + 1] = hi2(pg[j]);
            tp[D + 2 * j] = lo2(pb[j]);
            tp[D + 2 * j + 1] = hi2(pb[j]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) tp[2 * D + j] = pd[j];
    }
    if (tid >= CONSUMERS) __syncthreads();
    __syncthreads();
    const float* tpart = reinterpret_cast<const float*>(lsm_raw);
    for (int i = tid; i < 3 * D; i += blockDim.x) {
        float v = 0.0f;
#pragma unroll
        for (int t = 0; t < TEAMS; ++t) v += tpart[(size_t)t * 3 * D + i];
        part[(size_t)blockIdx.x * 3 * D + i] = v;
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// One warp per team for D = 768 and 1024: lane l owns the 8-column groups l, l + 32, ... (CPT =
// D / 32 columns; consecutive lanes read consecutive 16-byte pieces of a row), so a row's sums
// reduce inside the warp (no shared-memory exchange, no named barrier) and the per-row scalar
// work is spread over D / 32 columns per lane instead of 8.  Eight teams take alternate stages of
// a 4-row ring fed by one producer thread, as in ln_bwd_ring_kernel.  Arithmetic as
// ln_bwd_mx_kernel (row sums and dx with FP16 operands, FP32 accumulation) except the column sums:
// dgamma += dy xhat and dbeta += dy in FP32 from FP32 dy and xhat, so they match the FP32 column
// sums of the generic kernel; dbias += dx from the FP16 dx.
constexpr int kLnWarpTeams = 8;
template <int D, bool kRefFormula, bool kRes, bool kBias>
__global__ void __launch_bounds__(32 * kLnWarpTeams + 32, 1)
    ln_bwd_warp_kernel(half* __restrict__ dx, float* __restrict__ part, const half* __restrict__ dy,
                       const half* __restrict__ dres, const half* __restrict__ x, const half* __restrict__ g,
                       const float* __restrict__ mean, const float* __restrict__ rstd, int N, int stages, int* err) {
    using namespace tc;
    constexpr int R = kLnRows;
    static_assert(R == 4, "the row-sum butterfly below reduces 2 * 4 sums");
    constexpr int G = D / 256;                          // 8-column groups per lane
    static_assert(D % 256 == 0 && G <= 4, "D = 256 k, k <= 4");
    constexpr int TEAMS = kLnWarpTeams;
    constexpr int NT = kRes ? 3 : 2;
    constexpr uint32_t ROW_BYTES = D * 2;
    // At D = 1024 a stage also carries its rows' mean[R], rstd[R] (the consumers' own loads of them
    // were the leading stall); at D = 768 the consumers load them one stage ahead (measured faster).
    constexpr bool kStats = D >= 1024;
    constexpr uint32_t STATS_OFF = R * ROW_BYTES * NT;
    constexpr uint32_t STAGE_BYTES = STATS_OFF + (kStats ? 8 * R : 0);
    constexpr float kInvD = 1.0f / (float)D;
    extern __shared__ __align__(128) uint8_t lsm_raw[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(lsm_raw + (size_t)stages * STAGE_BYTES);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * stages);
    auto full = [&](int s) { return su32(bars + s); };
    auto empty = [&](int s) { return su32(bars + stages + s); };
    const int tid = threadIdx.x, lane = tid & 31, team = tid >> 5;
    if (tid == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    grid_dependency_wait();
    const int nstage = (N + R - 1) / R;

    if (team == TEAMS) {
        if (lane == 0) {                                // producer
            int k = 0;
            for (int gs = blockIdx.x; gs < nstage; gs += gridDim.x, ++k) {
                const int s = k % stages;
                if (!mbar_wait(empty(s), ((k / stages) & 1) ^ 1, abort_flag)) break;
                const int rows = min(R, N - gs * R);
                // a whole stage also brings its rows' mean and rstd (16 bytes each); a partial last
                // stage leaves them to the consumers' own loads
                mbar_expect_tx(full(s), (uint32_t)rows * ROW_BYTES * NT + (kStats && rows == R ? 8u * R : 0u));
                const uint32_t dst = su32(lsm_raw + (size_t)s * STAGE_BYTES);
                const size_t off = (size_t)gs * R * D;
                const uint32_t bytes = (uint32_t)rows * ROW_BYTES;
                bulk_load(dst, dy + off, bytes, full(s));
                bulk_load(dst + R * ROW_BYTES, x + off, bytes, full(s));
                if (kRes) bulk_load(dst + 2 * R * ROW_BYTES, dres + off, bytes, full(s));
                if (kStats && rows == R) {
                    bulk_load(dst + STATS_OFF, mean + (size_t)gs * R, 4u * R, full(s));
                    bulk_load(dst + STATS_OFF + 4u * R, rstd + (size_t)gs * R, 4u * R, full(s));
                }
            }
        }
    } else {
        uint32_t gam[G][4];
#pragma unroll
        for (int q = 0; q < G; ++q) {
            const uint4 gv = __ldg(reinterpret_cast<const uint4*>(g) + lane + 32 * q);
            gam[q][0] = gv.x; gam[q][1] = gv.y; gam[q][2] = gv.z; gam[q][3] = gv.w;
        }
        uint64_t pg[G][4], pb[G][4];
        float pd[G][8];
#pragma unroll
        for (int q = 0; q < G; ++q) {
#pragma unroll
            for (int j = 0; j < 4; ++j) { pg[q][j] = 0; pb[q][j] = 0; }
#pragma unroll
            for (int j = 0; j < 8; ++j) pd[q][j] = 0.f;
        }
        bool ok = true;
        const uint32_t ring = su32(lsm_raw);
        float nmr[R], nrr[R];
        if constexpr (!kStats) {
            const int row0 = (blockIdx.x + team * gridDim.x) * R;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                nmr[r] = row0 + r < N ? __ldg(mean + row0 + r) : 0.0f;
                nrr[r] = row0 + r < N ? __ldg(rstd + row0 + r) : 0.0f;
            }
        }
        for (int k = team; blockIdx.x + k * gridDim.x < nstage; k += TEAMS) {
            const int gs = blockIdx.x + k * gridDim.x;
            const int s = k % stages;
            const int row0 = gs * R;
            const int nrows = min(R, N - row0);
            float mr[R], rr[R];
            if constexpr (!kStats) {
                const int nrow0 = (blockIdx.x + (k + TEAMS) * gridDim.x) * R;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    mr[r] = nmr[r];
                    rr[r] = nrr[r];
                    nmr[r] = nrow0 + r < N ? __ldg(mean + nrow0 + r) : 0.0f;
                    nrr[r] = nrow0 + r < N ? __ldg(rstd + nrow0 + r) : 0.0f;
                }
            }
            ok = __all_sync(0xffffffffu, ok && mbar_wait(full(s), (k / stages) & 1, abort_flag));
            if (!kStats) {
            } else if (nrows == R) {
                const float4 m4 = lds128f(ring + (uint32_t)s * STAGE_BYTES + STATS_OFF);
                const float4 r4 = lds128f(ring + (uint32_t)s * STAGE_BYTES + STATS_OFF + 4u * R);
                mr[0] = m4.x; mr[1] = m4.y; mr[2] = m4.z; mr[3] = m4.w;
                rr[0] = r4.x; rr[1] = r4.y; rr[2] = r4.z; rr[3] = r4.w;
            } else {
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    mr[r] = r < nrows ? __ldg(mean + row0 + r) : 0.0f;
                    rr[r] = r < nrows ? __ldg(rstd + row0 + r) : 0.0f;
                }
            }
            const uint32_t sb = ring + (uint32_t)s * STAGE_BYTES + 16u * lane;
            float v8[2 * R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                float s1a = 0.f, s1b = 0.f, s2a = 0.f, s2b = 0.f;
                if (ok && r < nrows) {
#pragma unroll
                    for (int q = 0; q < G; ++q) {
                        const uint4 d = lds128(sb + r * ROW_BYTES + 512u * q);
                        const uint4 xv = lds128(sb + (R + r) * ROW_BYTES + 512u * q);
                        const uint32_t dd[4] = {d.x, d.y, d.z, d.w}, xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            mfma2(s1a, s1b, dd[j], gam[q][j]);
                            mfma2(s2a, s2b, h2u(__hmul2(u2h(dd[j]), u2h(gam[q][j]))), xx[j]);
                        }
                    }
                }
                v8[2 * r] = s1a + s1b;
                v8[2 * r + 1] = s2a + s2b;
            }
            // warp totals of the 8 sums (transposed butterfly): lane l ends with sum (l >> 2) & 7
            float tot;
            {
                const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
                float a4[4], a2[2];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float keep = b4 ? v8[i + 4] : v8[i], send = b4 ? v8[i] : v8[i + 4];
                    a4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
                }
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const float keep = b3 ? a4[i + 2] : a4[i], send = b3 ? a4[i] : a4[i + 2];
                    a2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
                }
                tot = (b2 ? a2[1] : a2[0]) + __shfl_xor_sync(0xffffffffu, b2 ? a2[0] : a2[1], 4);
                tot += __shfl_xor_sync(0xffffffffu, tot, 2);
                tot += __shfl_xor_sync(0xffffffffu, tot, 1);
            }
            float ts[2 * R];
#pragma unroll
            for (int q = 0; q < 2 * R; ++q) ts[q] = __shfl_sync(0xffffffffu, tot, 4 * q);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (ok && r < nrows) {
                    const float inv = rr[r], m = mr[r];
                    const float t1 = ts[2 * r], t2 = ts[2 * r + 1] - m * t1;
                    const float bh = -(kRefFormula ? inv : inv * inv) * t2 * kInvD;
                    const float c = -inv * t1 * kInvD;
                    const __half mhi = __float2half_rn(m);
                    const __half mlo = __float2half_rn(m - __half2float(mhi));
                    const __half2 mhi2 = __halves2half2(mhi, mhi), mlo2 = __halves2half2(mlo, mlo);
                    const __half2 inv2 = __float2half2_rn(inv), bh2 = __float2half2_rn(bh), c2 = __float2half2_rn(c);
                    const uint64_t iv2 = pk2(inv, inv), nmi2 = pk2(-m * inv, -m * inv);
                    half* dxr = dx + (size_t)(row0 + r) * D;
#pragma unroll
                    for (int q = 0; q < G; ++q) {
                        const uint4 d = lds128(sb + r * ROW_BYTES + 512u * q);
                        const uint4 xv = lds128(sb + (R + r) * ROW_BYTES + 512u * q);
                        uint4 rv = make_uint4(0u, 0u, 0u, 0u);
                        if (kRes) rv = lds128(sb + (2 * R + r) * ROW_BYTES + 512u * q);
                        const uint32_t dd[4] = {d.x, d.y, d.z, d.w}, xx[4] = {xv.x, xv.y, xv.z, xv.w};
                        const uint32_t rs[4] = {rv.x, rv.y, rv.z, rv.w};
                        uint64_t df[4], xf[4];
                        h8_to_p(d, df);
                        h8_to_p(xv, xf);
                        uint32_t o[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const __half2 xh = __hmul2(__hsub2(__hsub2(u2h(xx[j]), mhi2), mlo2), inv2);
                            const __half2 dg = __hmul2(u2h(dd[j]), u2h(gam[q][j]));
                            __half2 v = __hfma2(inv2, dg, __hfma2(bh2, xh, c2));
                            if (kRes) v = __hadd2(v, u2h(rs[j]));
                            o[j] = h2u(v);
                            pg[q][j] = pfma2(df[j], pfma2(xf[j], iv2, nmi2), pg[q][j]);   // dy (x inv - m inv)
                            pb[q][j] = padd2(pb[q][j], df[j]);
                            if (kBias) madd2(pd[q][2 * j], pd[q][2 * j + 1], o[j]);
                        }
                        reinterpret_cast<uint4*>(dxr)[lane + 32 * q] = make_uint4(o[0], o[1], o[2], o[3]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty(s));
        }
        if (!ok && lane == 0) atomicExch(err, RBK_ERR_TIMEOUT);
        __syncthreads();                                // the ring is consumed: reuse it for the partials
        float* tp = reinterpret_cast<float*>(lsm_raw) + (size_t)team * 3 * D;
#pragma unroll
        for (int q = 0; q < G; ++q) {
            const int c0 = 8 * (lane + 32 * q);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                tp[c0 + 2 * j] = lo2(pg[q][j]);
                tp[c0 + 2 * j + 1] = hi2(pg[q][j]);
                tp[D + c0 + 2 * j] = lo2(pb[q][j]);
                tp[D + c0 + 2 * j + 1] = hi2(pb[q][j]);
                tp[2 * D + c0 + 2 * j] = pd[q][2 * j];
                tp[2 * D + c0 + 2 * j + 1] = pd[q][2 * j + 1];
            }
        }
    }
    if (team == TEAMS) __syncthreads();
    __syncthreads();
    const float* tpart = reinterpret_cast<const float*>(lsm_raw);
    for (int i = tid; i < 3 * D; i += blockDim.x) {
        float v = 0.0f;
#pragma unroll
        for (int t = 0; t < TEAMS; ++t) v += tpart[(size_t)t * 3 * D + i];
        part[(size_t)blockIdx.x * 3 * D + i] = v;
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// cudaFuncSetAttribute once per (kernel, device, size): on every launch it would cost host time
// comparable to these kernels' own duration.
int ensure_smem(const void* fn, size_t smem) {
    static std::mutex mu;
    static std::vector<std::tuple<const void*, int, size_t>> done;
    int dev = 0;
    RBK_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lk(mu);
    for (const auto& t : done)
        if (std::get<0>(t) == fn && std::get<1>(t) == dev && std::get<2>(t) >= smem) return RBK_OK;
    RBK_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    done.emplace_back(fn, dev, smem);
    return RBK_OK;
}

template <int D, bool A, bool B, bool C>
int launch_bwd_warp(int blocks, int stages, size_t smem, cudaStream_t st, half* dx, float* part, const half* dy,
                    const half* dres, const half* x, const half* g, const float* mean, const float* rstd, int N,
                    int* err) {
    RBK_TRY(ensure_smem((const void*)ln_bwd_warp_kernel<D, A, B, C>, smem));
    RBK_CUDA(launch_pdl(ln_bwd_warp_kernel<D, A, B, C>, dim3(blocks), dim3(32 * kLnWarpTeams + 32), smem, st, dx, part,
                        dy, dres, x, g, mean, rstd, N, stages, err));
    return RBK_OK;
}

template <int D, bool A, bool B, bool C>
int launch_bwd_mx(int blocks, int threads, int stages, size_t smem, cudaStream_t st, half* dx, float* part,
                  const half* dy, const half* dres, const half* x, const half* g, const float* mean, const float* rstd,
                  int N, int* err) {
    RBK_TRY(ensure_smem((const void*)ln_bwd_mx_kernel<D, A, B, C>, smem));
    RBK_CUDA(launch_pdl(ln_bwd_mx_kernel<D, A, B, C>, dim3(blocks), dim3(threads), smem, st, dx, part, dy, dres, x, g,
                        mean, rstd, N, stages, err));
    return RBK_OK;
}

template <bool A, bool B, bool C>
int launch_bwd_ring(int blocks, int threads, int teams, int tpt, int stages, size_t smem, cudaStream_t st, half* dx,
                    float* part, const half* dy, const half* dres, const half* x, const half* g, const float* mean,
                    const float* rstd, int N, int D, int* err) {
    RBK_TRY(ensure_smem((const void*)ln_bwd_ring_kernel<A, B, C>, smem));
    RBK_CUDA(launch_pdl(ln_bwd_ring_kernel<A, B, C>, dim3(blocks), dim3(threads), smem, st, dx, part, dy, dres, x, g,
                        mean, rstd, N, D, teams, tpt, stages, err));
    return RBK_OK;
}

template <int NV>
int launch_fwd(int blocks, cudaStream_t st, half* y, float* mean, float* rstd, const half* x, const half* g,
               const half* b, int N, int D, float eps) {
    // the rows-in-flight variants (NV <= 4) walk rows with one wave of resident CTAs
    static int resident = 0;
    if (resident == 0) {
        int occ = 0, dev = 0, sms = 0;
        RBK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, ln_fwd_kernel<NV>, 256, 0));
        RBK_CUDA(cudaGetDevice(&dev));
        RBK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        resident = (occ > 0 ? occ : 1) * sms;
    }
    if (NV <= 8 && blocks > resident) blocks = resident;
    RBK_CUDA(launch_pdl(ln_fwd_kernel<NV>, dim3(blocks), dim3(256), 0, st, y, mean, rstd, x, g, b, N, D, eps));
    return RBK_OK;
}

template <bool A, bool B, bool C>
int launch_bwd(int blocks, int threads, int teams, size_t smem, cudaStream_t st, half* dx, float* part,
               const half* dy, const half* dres, const half* x, const half* g, const float* mean, const float* rstd,
               int N, int D) {
    if (smem > 48 * 1024) RBK_CUDA(cudaFuncSetAttribute(ln_bwd_kernel<A, B, C>,
                                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    ln_bwd_kernel<A, B, C><<<blocks, threads, smem, st>>>(dx, part, dy, dres, x, g, mean, rstd, N, D, teams);
    return RBK_OK;
}

}  // namespace
}  // namespace rbk

using namespace rbk;

extern "C" {

int rbk_ln_fwd(rbk_ctx* ctx, void* y, float* mean, float* rstd, const void* x, const void* gamma, const void* beta,
               int N, int D, float eps, void* stream) {
    RBK_REQUIRE(ctx && y && mean && rstd && x && gamma && beta, "rbk_ln_fwd: null pointer");
    RBK_REQUIRE(N > 0 && D > 0 && D % 8 == 0 && D <= 8192, "rbk_ln_fwd: need D %% 8 == 0 and D <= 8192 (D=%d)", D);
    RBK_REQUIRE(aligned16(y) && aligned16(x) && aligned16(gamma) && aligned16(beta),
                "rbk_ln_fwd: tensors must be 16-byte aligned");
    const int nv = (D / 8 + 31) / 32;
    const int rows_per_block = 8;
    int blocks = (N + rows_per_block - 1) / rows_per_block;
    blocks = blocks < ctx->num_sms * 16 ? blocks : ctx->num_sms * 16;
    cudaStream_t st = as_stream(stream);
    ProfScope prof(ctx, st, kCatLnFwd, 4.0 * N * D + 8.0 * N + 4.0 * D);
    auto Y = (half*)y;
    auto X = (const half*)x;
    auto G = (const half*)gamma;
    auto Bt = (const half*)beta;
    int rc;
    switch (nv) {
        case 1: rc = launch_fwd<1>(blocks, st, Y, mean, rstd, X, G, Bt, N, D, eps); break;
        case 2: rc = launch_fwd<2>(blocks, st, Y, mean, rstd, X, G, Bt, N, D, eps); break;
        case 3: rc = launch_fwd<3>(blocks, st, Y, mean, rstd, X, G, Bt, N, D, eps); break;
        case 4: rc = launch_fwd<4>(blocks, st, Y, mean, rstd, X, G, Bt, N, D, eps); break;
        case 5: case 6: rc = launch_fwd<6>(blocks, st, Y, mean, rstd, X, G, Bt, N, D, eps); break;
        case 7: case 8: rc = launch_fwd<8>(blocks, st, Y, mean, rstd, X, G, Bt, N, D, eps); break;
        case 9: case 10: case 11: case 12: rc = launch_fwd<12>(blocks, st, Y, mean, rstd, X, G, Bt, N, D, eps); break;
        case 13: case 14: case 15: case 16: rc = launch_fwd<16>(blocks, st, Y, mean, rstd, X, G, Bt, N, D, eps); break;
        default: rc = launch_fwd<32>(blocks, st, Y, mean, rstd, X, G, Bt, N, D, eps); break;
    }
    if (rc != RBK_OK) return rc;
    RBK_LAUNCHED("ln_fwd_kernel");
    return RBK_OK;
}

int rbk_ln_bwd(rbk_ctx* ctx, void* dx, float* dgamma, float* dbeta, float* dbias_out, const void* dy,
               const void* dres, const void* x, const void* gamma, const float* mean, const float* rstd, int N,
               int D, int flags, void* stream) {
    RBK_REQUIRE(ctx && dx && dgamma && dbeta && dy && x && gamma && mean && rstd, "rbk_ln_bwd: null pointer");
    RBK_REQUIRE(N > 0 && D > 0 && D % 8 == 0 && D <= 4096, "rbk_ln_bwd: need D %% 8 == 0 and D <= 4096 (D=%d)", D);
    RBK_REQUIRE(aligned16(dx) && aligned16(dy) && aligned16(x) && aligned16(gamma) && (!dres || aligned16(dres)),
                "rbk_ln_bwd: tensors must be 16-byte aligned");
    RBK_REQUIRE(aligned16(mean) && aligned16(rstd), "rbk_ln_bwd: mean / rstd must be 16-byte aligned");
    const int tpt = ((D / 8 + 31) / 32) * 32;            // threads per team
    int teams = 512 / tpt;
    teams = teams < 1 ? 1 : teams > kLnMaxTeams ? kLnMaxTeams : teams;
    const int threads = teams * tpt + 32;                // + the producer warp
    const int RS = kLnRows;                              // rows per ring stage (one team's)
    const size_t stage_bytes = (size_t)RS * D * 2 * (dres ? 3 : 2);
    int stages = (int)((200u << 10) / stage_bytes);
    stages = stages > 16 ? 16 : stages;
    RBK_REQUIRE(stages >= 2, "rbk_ln_bwd: row blocks too large for the shared-memory ring (D=%d)", D);
    const size_t smem = stages * stage_bytes + sizeof(float) * (size_t)teams * 2 * 2 * kLnRows * (tpt / 32) +
                        16 * (size_t)stages + 16;
    const int nstage = (N + RS - 1) / RS;
    int blocks = ctx->num_sms;                            // persistent: one CTA per SM
    if (blocks > nstage) blocks = nstage;
    void* ws;
    RBK_TRY(ctx_scratch(ctx, sizeof(float) * 3 * (size_t)D * blocks, &ws));
    float* part = (float*)ws;
    cudaStream_t st = as_stream(stream);
    // algorithmic bytes: x, dy, dx (+ dres) half rows, mean/rstd, gamma, FP32 column sums
    ProfScope prof(ctx, st, kCatLnBwd,
                   (double)N * D * (6.0 + (dres ? 2.0 : 0.0)) + 8.0 * N + (double)D * (2.0 + 8.0 + (dbias_out ? 4.0 : 0.0)));
    const bool ref = (flags & RBK_LN_REFERENCE_FORMULA) != 0;
    const bool res = dres != nullptr, bias = dbias_out != nullptr;
    auto DX = (half*)dx;
    auto DY = (const half*)dy;
    auto DR = (const half*)dres;
    auto X = (const half*)x;
    auto G = (const half*)gamma;
    int* err = ctx->tickets + kGemmError;
    static const bool generic_only = [] {
        const char* e = getenv("RBK_LN_GENERIC");
        return e && e[0] == '1';
    }();
    if (!generic_only && (D == 768 || D == 1024)) {
        // one warp per team: its own ring depth (the stage is 4 rows of every tensor)
        const size_t wstage = (size_t)kLnRows * D * 2 * (dres ? 3 : 2) + (D >= 1024 ? 8 * kLnRows : 0);   // + stats
        int wst = (int)((200u << 10) / wstage);
        wst = wst > 16 ? 16 : wst;
        const size_t wsmem = wst * wstage + 16 * (size_t)wst + 16;
        RBK_REQUIRE(wsmem >= sizeof(float) * 3 * (size_t)D * kLnWarpTeams, "rbk_ln_bwd: partial area");
#define RBK_LN_W(D_, R_, S_, B_) \
    RBK_TRY((launch_bwd_warp<D_, R_, S_, B_>(blocks, wst, wsmem, st, DX, part, DY, DR, X, G, mean, rstd, N, err)))
#define RBK_LN_W_D(D_)                                                                                        \
    if (ref) {                                                                                                \
        if (res) { if (bias) RBK_LN_W(D_, true, true, true); else RBK_LN_W(D_, true, true, false); }           \
        else { if (bias) RBK_LN_W(D_, true, false, true); else RBK_LN_W(D_, true, false, false); }            \
    } else {                                                                                                  \
        if (res) { if (bias) RBK_LN_W(D_, false, true, true); else RBK_LN_W(D_, false, true, false); }         \
        else { if (bias) RBK_LN_W(D_, false, false, true); else RBK_LN_W(D_, false, false, false); }          \
    }
        if (D == 768) { RBK_LN_W_D(768) }
        else { RBK_LN_W_D(1024) }
#undef RBK_LN_W_D
#undef RBK_LN_W
        RBK_LAUNCHED("ln_bwd_warp_kernel");
    } else if (!generic_only && D == 2048) {
        // the specialised mixed-precision kernel: same teams, ring and launch shape
#define RBK_LN_MX(D_, R_, S_, B_)                                                                                \
    RBK_TRY((launch_bwd_mx<D_, R_, S_, B_>(blocks, threads, stages, smem, st, DX, part, DY, DR, X, G, mean, rstd, N, \
                                           err)))
#define RBK_LN_MX_D(D_)                                                                                       \
    if (ref) {                                                                                                \
        if (res) { if (bias) RBK_LN_MX(D_, true, true, true); else RBK_LN_MX(D_, true, true, false); }         \
        else { if (bias) RBK_LN_MX(D_, true, false, true); else RBK_LN_MX(D_, true, false, false); }          \
    } else {                                                                                                  \
        if (res) { if (bias) RBK_LN_MX(D_, false, true, true); else RBK_LN_MX(D_, false, true, false); }       \
        else { if (bias) RBK_LN_MX(D_, false, false, true); else RBK_LN_MX(D_, false, false, false); }        \
    }
        RBK_LN_MX_D(2048)
#undef RBK_LN_MX_D
#undef RBK_LN_MX
        RBK_LAUNCHED("ln_bwd_mx_kernel");
    } else {
#define RBK_LN_BWD(R_, S_, B_)                                                                                  \
    RBK_TRY((launch_bwd_ring<R_, S_, B_>(blocks, threads, teams, tpt, stages, smem, st, DX, part, DY, DR, X, G, \
                                         mean, rstd, N, D, err)))
    if (ref) {
        if (res) { if (bias) RBK_LN_BWD(true, true, true); else RBK_LN_BWD(true, true, false); }
        else { if (bias) RBK_LN_BWD(true, false, true); else RBK_LN_BWD(true, false, false); }
    } else {
        if (res) { if (bias) RBK_LN_BWD(false, true, true); else RBK_LN_BWD(false, true, false); }
        else { if (bias) RBK_LN_BWD(false, false, true); else RBK_LN_BWD(false, false, false); }
    }
#undef RBK_LN_BWD
    RBK_LAUNCHED("ln_bwd_ring_kernel");
    }
    {
        // programmatic dependent launch: the reduce's launch overlaps the main pass's tail
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3((D + 31) / 32, bias ? 3 : 2);
        lc.blockDim = dim3(1024);
        lc.stream = st;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        lc.attrs = at;
        lc.numAttrs = 1;
        const float* cpart = part;
        RBK_CUDA(cudaLaunchKernelEx(&lc, ln_bwd_reduce_kernel, dgamma, dbeta, dbias_out, cpart, blocks, D));
    }
    RBK_LAUNCHED("ln_bwd_reduce_kernel");
    return RBK_OK;
}

}  // extern "C"

// ----------------------------------------------------------------------------
// LayerNorm backward for callers that cannot allocate device memory.
//
// Some callers own every byte of device memory through their own pool (the
// reference trainer reserves a fixed arena up front, src/cuda_kernels.cuh:46-57),
// or cannot afford an allocation — cudaMalloc / cudaFree synchronise the device
// — inside their step loop.  They cannot create an rbk_ctx either, because the
// context allocates its flags and scratch.  This variant needs no context: its
// column partials live in the fixed array below, which the library reserves
// once per GPU that loads it and holds until the process exits.
// ----------------------------------------------------------------------------
#include <mutex>

namespace rbk {
namespace {

constexpr size_t kNoAllocScratchBytes = RBK_LN_BWD_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) float g_ln_bwd_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {};   // device address of the array, per device
int g_noalloc_sms[kNoAllocMaxDevices] = {};

// Set-up on the first call on a device (with that device current): the host
// name of a __device__ array is only a host-side stand-in, so the kernel must
// be given the address the runtime reports for this device.
int noalloc_setup(int* dev_out, float** ptr, int* sms) {
    int dev = 0;
    RBK_CUDA(cudaGetDevice(&dev));
    RBK_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, "rbk_ln_bwd_noalloc: device %d beyond %d", dev,
                kNoAllocMaxDevices);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        cudaDeviceProp prop;
        RBK_CUDA(cudaGetDeviceProperties(&prop, dev));
        if (prop.major != 10 || prop.minor != 0) {
            set_error("librbk is built for sm_100a (B200); device %d is sm_%d%d", dev, prop.major, prop.minor);
            return RBK_ERR_UNSUPPORTED;
        }
        void* p = nullptr;
        RBK_CUDA(cudaGetSymbolAddress(&p, g_ln_bwd_noalloc_scratch));
        g_noalloc_sms[dev] = prop.multiProcessorCount;
        g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    *dev_out = dev;
    *ptr = g_noalloc_ptr[dev];
    *sms = g_noalloc_sms[dev];
    return RBK_OK;
}

}  // namespace
}  // namespace rbk

extern "C" int rbk_ln_bwd_noalloc(void* dx, float* dgamma, float* dbeta, float* dbias_out, const void* dy,
                                  const void* dres, const void* x, const void* gamma, const float* mean,
                                  const float* rstd, int N, int D, int flags, void* stream) {
    RBK_REQUIRE(dx && dgamma && dbeta && dy && x && gamma && mean && rstd, "rbk_ln_bwd_noalloc: null pointer");
    RBK_REQUIRE(N > 0 && D > 0 && D % 8 == 0 && D <= 4096,
                "rbk_ln_bwd_noalloc: need D %% 8 == 0 and D <= 4096 (D=%d)", D);
    RBK_REQUIRE(aligned16(dx) && aligned16(dy) && aligned16(x) && aligned16(gamma) && (!dres || aligned16(dres)),
                "rbk_ln_bwd_noalloc: tensors must be 16-byte aligned");
    int dev = 0, sms = 0;
    float* part = nullptr;
    RBK_TRY(noalloc_setup(&dev, &part, &sms));
    if (stream) {
        // the array's address is per device: a stream of another GPU would get the wrong one
        int sdev = -1;
        RBK_CUDA(cudaStreamGetDevice(as_stream(stream), &sdev));
        RBK_REQUIRE(sdev == dev, "rbk_ln_bwd_noalloc: the stream belongs to device %d, the current device is %d",
                    sdev, dev);
    }
    // A separate kernel from rbk_ln_bwd's ring (scalar FP32 arithmetic, one team per row group,
    // no timeout word): the results agree with rbk_ln_bwd to rounding, not bit for bit.
    const int tpt = ((D / 8 + 31) / 32) * 32;
    int teams = 512 / tpt;
    teams = teams < 1 ? 1 : teams > kLnMaxTeams ? kLnMaxTeams : teams;
    const int threads = teams * tpt;
    const int ngroups = (N + kLnRows - 1) / kLnRows;
    int blocks = sms;
    const int need = (ngroups + teams - 1) / teams;
    if (blocks > need) blocks = need;
    const size_t scratch = sizeof(float) * 3 * (size_t)D * blocks;
    if (scratch > kNoAllocScratchBytes) {
        set_error("rbk_ln_bwd_noalloc: needs %zu bytes of scratch (3 x D=%d x %d CTAs x 4 B) but the fixed "
                  "array holds %zu; use rbk_ln_bwd for this size",
                  scratch, D, blocks, kNoAllocScratchBytes);
        return RBK_ERR_INVALID;
    }
    const size_t smem = sizeof(float) * ((size_t)2 * teams * 2 * kLnRows * (tpt / 32) + (size_t)teams * 3 * D);
    cudaStream_t st = as_stream(stream);
    const bool ref = (flags & RBK_LN_REFERENCE_FORMULA) != 0;
    const bool res = dres != nullptr, bias = dbias_out != nullptr;
    auto DX = (half*)dx;
    auto DY = (const half*)dy;
    auto DR = (const half*)dres;
    auto X = (const half*)x;
    auto G = (const half*)gamma;
#define RBK_LN_BWD(R_, S_, B_) \
    RBK_TRY((launch_bwd<R_, S_, B_>(blocks, threads, teams, smem, st, DX, part, DY, DR, X, G, mean, rstd, N, D)))
    if (ref) {
        if (res) { if (bias) RBK_LN_BWD(true, true, true); else RBK_LN_BWD(true, true, false); }
        else { if (bias) RBK_LN_BWD(true, false, true); else RBK_LN_BWD(true, false, false); }
    } else {
        if (res) { if (bias) RBK_LN_BWD(false, true, true); else RBK_LN_BWD(false, true, false); }
        else { if (bias) RBK_LN_BWD(false, false, true); else RBK_LN_BWD(false, false, false); }
    }
#undef RBK_LN_BWD
    RBK_LAUNCHED("ln_bwd_kernel (no-alloc)");
    dim3 rg((D + 31) / 32, bias ? 3 : 2);
    ln_bwd_reduce_kernel<<<rg, 1024, 0, st>>>(dgamma, dbeta, dbias_out, part, blocks, D);
    RBK_LAUNCHED("ln_bwd_reduce_kernel (no-alloc)");
    return RBK_OK;
}
