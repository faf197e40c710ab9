// attn.cu — causal flash attention forward / backward (d_head 64 or 128).
//
// Replaces the reference's materialised attention (per-(b,h) cuBLAS score
// GEMMs, apply_causal_mask_fp32, softmax_fp32_forward into an FP32 [B,H,T,T]
// buffer, src/model.cu:262-286) and adds the backward the reference never runs
// (src/model.cu:387-397).  Scores are scaled by 1/sqrt(d_h) and masked
// causally as src/cpu_model.cpp:148-170 (the reference's -1e9 mask becomes an
// exact zero probability here).
//
// Tiles of 64 queries x 64 keys, 4 warps of 16 rows, FP16 operands from
// 128-byte-row shared tiles with a 16-byte XOR swizzle (conflict-free
// ldmatrix), FP32 accumulation, online softmax in the exp2 domain, LSE saved.
// Backward (FlashAttention-2 scheme): one CTA per 64-key block walks the
// query blocks at and below the diagonal, accumulates dK / dV in registers and
// adds dQ into an FP32 buffer with vector reductions; a final pass converts dQ
// and produces the bq / bk / bv gradient column sums.
//
// Tensor-core path: mma.sync m16n8k16 (this kernel predates the tcgen05
// version planned for attention; the GEMMs of the model run on tcgen05).
#include "common.cuh"

namespace rbk {

// tcgen05 main backward pass for d_head 64 / 128, S % 64 == 0 (attn_bwd_tc.cu).
// dq_sem (deterministic mode): zeroed ints [B*H, S/64] that order the dQ additions.
int attn_bwd_tc(rbk_ctx* ctx, void* dqkv, float* dq_acc, const void* qkv, const void* dout, const float* NL2,
                const float* Dot, int B, int S, int H, int dh, float scale, cudaStream_t st, int* dq_sem);

namespace attn {

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void ldsm4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(a));
}
__device__ __forceinline__ void ldsm4t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(a));
}
__device__ __forceinline__ void mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ void cp16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void red2(float* p, float a, float b) {
    asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(a), "f"(b) : "memory");
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int BLK = 64;

// Byte offset of element (r, c) (c a multiple of 8) in a [64][W] half tile
// whose 16-byte chunks are XOR-swizzled by the row index.
template <int W>
__device__ __forceinline__ uint32_t toff(int r, int c) {
    return (uint32_t)(r * W * 2 + (((c >> 3) ^ (r & 7)) << 4));
}

// 64 rows x W halves from global (row stride ld elements) into a swizzled tile.
template <int W>
__device__ __forceinline__ void load_tile(uint32_t s, const half* g, int ld, int tid) {
    constexpr int CH = W / 8;
#pragma unroll
    for (int i = tid; i < BLK * CH; i += 128) {
        const int r = i / CH, c = i % CH;
        cp16(s + toff<W>(r, c * 8), g + (size_t)r * ld + c * 8);
    }
}

// ------------------------------------------------------------------ forward --
template <int HD>
__global__ void __launch_bounds__(128) flash_fwd_kernel(half* __restrict__ O, float* __restrict__ LSE,
                                                        const half* __restrict__ qkv, int S, int H, float scale_log2) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int nqb = S / BLK;
    const int qb = nqb - 1 - (int)blockIdx.x;   // longest rows first
    const int bh = blockIdx.y, b = bh / H, h = bh % H;
    const int ld = 3 * H * HD;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, tig = lane & 3;
    const half* Qg = qkv + ((size_t)b * S + qb * BLK) * ld + h * HD;
    const half* Kg = qkv + (size_t)b * S * ld + H * HD + h * HD;
    const half* Vg = qkv + (size_t)b * S * ld + 2 * H * HD + h * HD;
    constexpr uint32_t TB = BLK * HD * 2;
    const uint32_t sQ = saddr(sm), sK = sQ + TB, sV = sK + 2 * TB;

    load_tile<HD>(sQ, Qg, ld, tid);
    load_tile<HD>(sK, Kg, ld, tid);
    load_tile<HD>(sV, Vg, ld, tid);
    cp_commit();

    float o[HD / 8][4];
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.0f, 0.0f};
    uint32_t qf[HD / 16][4];
    const int nkv = qb + 1;
    for (int j = 0; j < nkv; ++j) {
        if (j + 1 < nkv) {
            load_tile<HD>(sK + ((j + 1) & 1) * TB, Kg + (size_t)(j + 1) * BLK * ld, ld, tid);
            load_tile<HD>(sV + ((j + 1) & 1) * TB, Vg + (size_t)(j + 1) * BLK * ld, ld, tid);
            cp_commit();
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();
        if (j == 0) {
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk)
                ldsm4(sQ + toff<HD>(warp * 16 + (lane & 15), kk * 16 + 8 * (lane >> 4)), qf[kk][0], qf[kk][1],
                      qf[kk][2], qf[kk][3]);
        }
        const uint32_t kb = sK + (j & 1) * TB, vb = sV + (j & 1) * TB;
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t b0, b1, b2, b3;
                ldsm4(kb + toff<HD>(np * 16 + (lane & 7) + 8 * (lane >> 4), kk * 16 + 8 * ((lane >> 3) & 1)), b0, b1,
                      b2, b3);
                mma(s[2 * np], qf[kk], b0, b1);
                mma(s[2 * np + 1], qf[kk], b2, b3);
            }
        }
        const bool diag = (j == qb);
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float x = s[nt][e] * scale_log2;
                if (diag) {
                    const int row = warp * 16 + g + 8 * (e >> 1);
                    const int col = nt * 8 + 2 * tig + (e & 1);
                    if (col > row) x = -INFINITY;
                }
                s[nt][e] = x;
                mx[e >> 1] = fmaxf(mx[e >> 1], x);
            }
        float corr[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
            const float mn = fmaxf(mrow[r], mx[r]);
            corr[r] = ex2(mrow[r] - mn);
            mrow[r] = mn;
            lrow[r] *= corr[r];
        }
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
            o[i][0] *= corr[0]; o[i][1] *= corr[0];
            o[i][2] *= corr[1]; o[i][3] *= corr[1];
        }
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float p = ex2(s[nt][e] - mrow[e >> 1]);
                s[nt][e] = p;
                lrow[e >> 1] += p;
            }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t a[4] = {pack(s[2 * kk][0], s[2 * kk][1]), pack(s[2 * kk][2], s[2 * kk][3]),
                             pack(s[2 * kk + 1][0], s[2 * kk + 1][1]), pack(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
            for (int dp = 0; dp < HD / 16; ++dp) {
                uint32_t b0, b1, b2, b3;
                ldsm4t(vb + toff<HD>(kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1), dp * 16 + 8 * (lane >> 4)), b0, b1,
                       b2, b3);
                mma(o[2 * dp], a, b0, b1);
                mma(o[2 * dp + 1], a, b2, b3);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
    }
    const int D = H * HD;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int row = qb * BLK + warp * 16 + g + 8 * r;
        const float inv = 1.0f / lrow[r];
        half* orow = O + ((size_t)b * S + row) * D + h * HD;
#pragma unroll
        for (int nt = 0; nt < HD / 8; ++nt)
            *reinterpret_cast<__half2*>(orow + nt * 8 + 2 * tig) =
                __floats2half2_rn(o[nt][2 * r] * inv, o[nt][2 * r + 1] * inv);
        if (tig == 0) LSE[(size_t)bh * S + row] = (mrow[r] + __log2f(lrow[r])) * kLn2;
    }
}

// ------------------------------------------------------------------ backward --

// Pre and post passes share one row-block layout: block (TX, TY) with TX a
// multiple of 32 (one warp never spans two row teams), thread (x, y) owns the
// 8 columns c8 = blockIdx.x * TX + x and the rows r0 + y, r0 + y + TY, ... of
// its CTA's row block [r0, r1).  Four rows are loaded before any is used, so a
// thread keeps 4 x 32 bytes in flight.  Column sums (bias gradients) fold the
// TY row teams in shared memory and leave one partial row per CTA in
// part[blockIdx.y][0, D); attn_bias_reduce_kernel adds the partial rows in a
// fixed order (no atomics: every CTA would otherwise add into the same D
// addresses).
constexpr int kRowUnroll = 4;

// Fold acc[8] over the row teams of the CTA into part[c8 * 8, +8).  red holds
// blockDim.x * blockDim.y * 8 floats.  Every thread of the CTA calls it.
__device__ __forceinline__ void fold_column_sums(const float (&acc)[8], float* __restrict__ part, int c8, bool col_ok,
                                                 float* red) {
    const int t = threadIdx.y * blockDim.x + threadIdx.x;
    float4* r4 = reinterpret_cast<float4*>(red);
    r4[2 * t] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    r4[2 * t + 1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    __syncthreads();
    if (threadIdx.y == 0 && col_ok) {
        float4 a = r4[2 * t], b = r4[2 * t + 1];
        for (int y = 1; y < (int)blockDim.y; ++y) {
            const int u = y * blockDim.x + threadIdx.x;
            const float4 c = r4[2 * u], d = r4[2 * u + 1];
            a.x += c.x; a.y += c.y; a.z += c.z; a.w += c.w;
            b.x += d.x; b.y += d.y; b.z += d.z; b.w += d.w;
        }
        float4* out = reinterpret_cast<float4*>(part + (size_t)c8 * 8);
        out[0] = a;
        out[1] = b;
    }
}

// Dot[bh, s] = sum_d dO[s, d] O[s, d]  and zero the FP32 dQ accumulator; with
// NL2 also NL2[bh, s] = -LSE[bh, s] * log2 e (the tcgen05 main pass reads it);
// with vpart also the column sums of dO, one partial row per CTA (the v-bias
// gradient of the tcgen05 path, whose main pass writes no bias terms:
// sum_keys dV = sum_queries dO because every row of P sums to 1).  The HD/8
// threads of a head reduce the dot by shuffles (adjacent lanes of one warp:
// HD/8 divides 32 and TX is a multiple of 32).
template <int HD>
__global__ void __launch_bounds__(512, 2)
    flash_bwd_pre_kernel(float* __restrict__ Dot, float* __restrict__ dq_acc, float* __restrict__ NL2,
                         float* __restrict__ vpart, const float* __restrict__ LSE, const half* __restrict__ O,
                         const half* __restrict__ dO, int BS, int S, int H, int rows_per_block, int* __restrict__ sem,
                         int nsem) {
    grid_dependency_sync();
    if (sem) {                           // the main pass's dQ ordering counters start at zero
        const int nt = blockDim.x * blockDim.y * gridDim.x * gridDim.y;
        const int id = ((blockIdx.y * gridDim.x + blockIdx.x) * blockDim.y + threadIdx.y) * blockDim.x + threadIdx.x;
        for (int i = id; i < nsem; i += nt) sem[i] = 0;
    }
    __shared__ __align__(16) float red[512 * 8];
    constexpr int G = HD / 8;            // chunks per (row, head)
    const int D = H * HD;
    const int TY = blockDim.y;
    const int c8 = blockIdx.x * blockDim.x + threadIdx.x;
    const bool col_ok = c8 * 8 < D;
    const int h = c8 / G;
    const int r0 = blockIdx.y * rows_per_block, r1 = min(BS, r0 + rows_per_block);
    float accv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // warp-uniform trip count (a warp lies in one row team)
    for (int rb = r0 + threadIdx.y; rb < r1; rb += kRowUnroll * TY) {
        uint4 a[kRowUnroll], d[kRowUnroll];
#pragma unroll
        for (int u = 0; u < kRowUnroll; ++u) {
            const int r = rb + u * TY;
            if (col_ok && r < r1) {
                a[u] = __ldg(reinterpret_cast<const uint4*>(O + (size_t)r * D) + c8);
                d[u] = __ldg(reinterpret_cast<const uint4*>(dO + (size_t)r * D) + c8);
            } else {
                a[u] = make_uint4(0u, 0u, 0u, 0u);
                d[u] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
#pragma unroll
        for (int u = 0; u < kRowUnroll; ++u) {
            const int r = rb + u * TY;
            float fa[8], fd[8];
            h8_to_f(a[u], fa);
            h8_to_f(d[u], fd);
            float acc = 0.0f;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                acc += fa[k] * fd[k];
                accv[k] += fd[k];
            }
#pragma unroll
            for (int o = 1; o < G; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (col_ok && r < r1) {
                float4* z = reinterpret_cast<float4*>(dq_acc + (size_t)r * D) + 2 * c8;
                z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
                z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
                if ((threadIdx.x & (G - 1)) == 0) {
                    const int b = r / S, s = r % S;
                    const size_t idx = ((size_t)b * H + h) * S + s;
                    Dot[idx] = acc;
                    if (NL2) NL2[idx] = -LSE[idx] * kLog2e;
                }
            }
        }
    }
    if (vpart) fold_column_sums(accv, vpart + (size_t)blockIdx.y * D, c8, col_ok, red);
}

template <int HD>
__global__ void __launch_bounds__(128) flash_bwd_kernel(half* __restrict__ dqkv, float* __restrict__ dq_acc,
                                                        float* __restrict__ dbias, const half* __restrict__ qkv,
                                                        const half* __restrict__ dO, const float* __restrict__ LSE,
                                                        const float* __restrict__ Dot, int S, int H, float scale,
                                                        float scale_log2) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int nkb = S / BLK;
    const int kb_idx = (int)blockIdx.x;          // low key blocks see the most query blocks: go first
    const int bh = blockIdx.y, b = bh / H, h = bh % H;
    const int ld = 3 * H * HD, D = H * HD;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, tig = lane & 3;
    constexpr uint32_t TB = BLK * HD * 2;
    const uint32_t sK = saddr(sm), sV = sK + TB, sQ = sV + TB, sdO = sQ + 2 * TB, sdS = sdO + 2 * TB;
    float* sL = reinterpret_cast<float*>(sm + 6 * TB + BLK * BLK * 2);   // [2][64] lse (log2 domain)
    float* sD = sL + 2 * BLK;                                            // [2][64] Dot
    const half* base = qkv + (size_t)b * S * ld;
    const half* Kg = base + (size_t)kb_idx * BLK * ld + H * HD + h * HD;
    const half* Vg = base + (size_t)kb_idx * BLK * ld + 2 * H * HD + h * HD;
    const half* Qg = base + h * HD;
    const half* dOg = dO + (size_t)b * S * D + h * HD;
    const float* Lg = LSE + (size_t)bh * S;
    const float* Dg = Dot + (size_t)bh * S;

    load_tile<HD>(sK, Kg, ld, tid);
    load_tile<HD>(sV, Vg, ld, tid);
    auto load_q = [&](int qi, int buf) {
        load_tile<HD>(sQ + buf * TB, Qg + (size_t)qi * BLK * ld, ld, tid);
        load_tile<HD>(sdO + buf * TB, dOg + (size_t)qi * BLK * D, D, tid);
        if (tid < BLK) {
            sL[buf * BLK + tid] = Lg[qi * BLK + tid] * kLog2e;
            sD[buf * BLK + tid] = Dg[qi * BLK + tid];
        }
    };
    load_q(kb_idx, 0);
    cp_commit();

    float dv[HD / 8][4], dk[HD / 8][4];
#pragma unroll
    for (int i = 0; i < HD / 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) dv[i][e] = dk[i][e] = 0.0f;
    const int kr = warp * 16;   // this warp's 16 keys inside the block

    for (int qi = kb_idx; qi < nkb; ++qi) {
        const int buf = (qi - kb_idx) & 1;
        if (qi + 1 < nkb) {
            load_q(qi + 1, buf ^ 1);
            cp_commit();
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();
        const uint32_t q_s = sQ + buf * TB, do_s = sdO + buf * TB;
        const float* lq = sL + buf * BLK;
        const float* dq = sD + buf * BLK;
        // S^T = K_w Q^T and dP^T = V_w dO^T  (16 keys x 64 queries each)
        float st[8][4], dpt[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) st[i][e] = dpt[i][e] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
            uint32_t ka[4], va[4];
            ldsm4(sK + toff<HD>(kr + (lane & 15), kk * 16 + 8 * (lane >> 4)), ka[0], ka[1], ka[2], ka[3]);
            ldsm4(sV + toff<HD>(kr + (lane & 15), kk * 16 + 8 * (lane >> 4)), va[0], va[1], va[2], va[3]);
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                const int rr = np * 16 + (lane & 7) + 8 * (lane >> 4), cc = kk * 16 + 8 * ((lane >> 3) & 1);
                uint32_t b0, b1, b2, b3;
                ldsm4(q_s + toff<HD>(rr, cc), b0, b1, b2, b3);
                mma(st[2 * np], ka, b0, b1);
                mma(st[2 * np + 1], ka, b2, b3);
                ldsm4(do_s + toff<HD>(rr, cc), b0, b1, b2, b3);
                mma(dpt[2 * np], va, b0, b1);
                mma(dpt[2 * np + 1], va, b2, b3);
            }
        }
        // P^T and dS^T = P^T (dP^T - Dot[q])
        const bool diag = (qi == kb_idx);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = kr + g + 8 * (e >> 1);
                const int q = nt * 8 + 2 * tig + (e & 1);
                float p = ex2(st[nt][e] * scale_log2 - lq[q]);
                if (diag && key > q) p = 0.0f;
                st[nt][e] = p;
                dpt[nt][e] = p * (dpt[nt][e] - dq[q]);
            }
        // dV += P^T dO ; dK += dS^T Q     (contraction over the 64 queries)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t pa[4] = {pack(st[2 * kk][0], st[2 * kk][1]), pack(st[2 * kk][2], st[2 * kk][3]),
                              pack(st[2 * kk + 1][0], st[2 * kk + 1][1]), pack(st[2 * kk + 1][2], st[2 * kk + 1][3])};
            uint32_t sa[4] = {pack(dpt[2 * kk][0], dpt[2 * kk][1]), pack(dpt[2 * kk][2], dpt[2 * kk][3]),
                              pack(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]),
                              pack(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3])};
#pragma unroll
            for (int dp = 0; dp < HD / 16; ++dp) {
                const int rr = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1), cc = dp * 16 + 8 * (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldsm4t(do_s + toff<HD>(rr, cc), b0, b1, b2, b3);
                mma(dv[2 * dp], pa, b0, b1);
                mma(dv[2 * dp + 1], pa, b2, b3);
                ldsm4t(q_s + toff<HD>(rr, cc), b0, b1, b2, b3);
                mma(dk[2 * dp], sa, b0, b1);
                mma(dk[2 * dp + 1], sa, b2, b3);
            }
        }
        // dS^T -> shared [64 keys][64 queries] (half)
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int key = kr + g + 8 * r;
                const uint32_t a = sdS + toff<BLK>(key, nt * 8) + 4 * tig;
                const uint32_t v = pack(dpt[nt][2 * r], dpt[nt][2 * r + 1]);
                asm volatile("st.shared.b32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
            }
        __syncthreads();
        // dQ(16 queries of this warp) += dS K   (contraction over the 64 keys)
        float dqa[HD / 8][4];
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) dqa[i][0] = dqa[i][1] = dqa[i][2] = dqa[i][3] = 0.0f;
        const int qr = warp * 16;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t a[4];
            const int mi = lane >> 3;
            ldsm4t(sdS + toff<BLK>(kk * 16 + (lane & 7) + 8 * (mi >> 1), qr + 8 * (mi & 1)), a[0], a[1], a[2], a[3]);
#pragma unroll
            for (int dp = 0; dp < HD / 16; ++dp) {
                uint32_t b0, b1, b2, b3;
                ldsm4t(sK + toff<HD>(kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1), dp * 16 + 8 * (lane >> 4)), b0, b1,
                       b2, b3);
                mma(dqa[2 * dp], a, b0, b1);
                mma(dqa[2 * dp + 1], a, b2, b3);
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float* dst = dq_acc + ((size_t)b * S + qi * BLK + qr + g + 8 * r) * D + h * HD + 2 * tig;
#pragma unroll
            for (int nt = 0; nt < HD / 8; ++nt) red2(dst + nt * 8, dqa[nt][2 * r] * scale, dqa[nt][2 * r + 1] * scale);
        }
        __syncthreads();
    }
    // dK (scaled), dV -> dqkv ; bias gradients of k and v (column sums over keys)
    float ck[HD / 8][2], cv[HD / 8][2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int key = kb_idx * BLK + kr + g + 8 * r;
        half* krow = dqkv + ((size_t)b * S + key) * ld + H * HD + h * HD;
        half* vrow = dqkv + ((size_t)b * S + key) * ld + 2 * H * HD + h * HD;
#pragma unroll
        for (int nt = 0; nt < HD / 8; ++nt) {
            const float k0 = dk[nt][2 * r] * scale, k1 = dk[nt][2 * r + 1] * scale;
            *reinterpret_cast<__half2*>(krow + nt * 8 + 2 * tig) = __floats2half2_rn(k0, k1);
            *reinterpret_cast<__half2*>(vrow + nt * 8 + 2 * tig) = __floats2half2_rn(dv[nt][2 * r], dv[nt][2 * r + 1]);
            if (r == 0) { ck[nt][0] = k0; ck[nt][1] = k1; cv[nt][0] = dv[nt][0]; cv[nt][1] = dv[nt][1]; }
            else { ck[nt][0] += k0; ck[nt][1] += k1; cv[nt][0] += dv[nt][2]; cv[nt][1] += dv[nt][3]; }
        }
    }
    if (dbias) {
#pragma unroll
        for (int nt = 0; nt < HD / 8; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e)
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) {
                    ck[nt][e] += __shfl_xor_sync(0xffffffffu, ck[nt][e], o);
                    cv[nt][e] += __shfl_xor_sync(0xffffffffu, cv[nt][e], o);
                }
        if (g == 0) {
#pragma unroll
            for (int nt = 0; nt < HD / 8; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    atomicAdd(dbias + H * HD + h * HD + nt * 8 + 2 * tig + e, ck[nt][e]);
                    atomicAdd(dbias + 2 * H * HD + h * HD + nt * 8 + 2 * tig + e, cv[nt][e]);
                }
        }
    }
}

// dqkv[:, q block] = half(dq_acc); with qpart also the column sums of dq_acc,
// one partial row per CTA (the q-bias gradient).  Row-block layout as in the
// pre pass.
__global__ void __launch_bounds__(512, 2)
    flash_bwd_post_kernel(half* __restrict__ dqkv, float* __restrict__ qpart, const float* __restrict__ dq_acc, int BS,
                          int D, int rows_per_block) {
    grid_dependency_sync();
    __shared__ __align__(16) float red[512 * 8];
    const int TY = blockDim.y;
    const int c8 = blockIdx.x * blockDim.x + threadIdx.x;
    const bool col_ok = c8 * 8 < D;
    const int r0 = blockIdx.y * rows_per_block, r1 = min(BS, r0 + rows_per_block);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (col_ok) {
        for (int rb = r0 + threadIdx.y; rb < r1; rb += kRowUnroll * TY) {
            float4 v[kRowUnroll][2];
#pragma unroll
            for (int u = 0; u < kRowUnroll; ++u) {
                const int r = rb + u * TY;
                if (r < r1) {
                    const float4* src = reinterpret_cast<const float4*>(dq_acc + (size_t)r * D) + 2 * c8;
                    v[u][0] = __ldg(src);
                    v[u][1] = __ldg(src + 1);
                } else {
                    v[u][0] = make_float4(0.f, 0.f, 0.f, 0.f);
                    v[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
#pragma unroll
            for (int u = 0; u < kRowUnroll; ++u) {
                const int r = rb + u * TY;
                const float x[8] = {v[u][0].x, v[u][0].y, v[u][0].z, v[u][0].w,
                                    v[u][1].x, v[u][1].y, v[u][1].z, v[u][1].w};
#pragma unroll
                for (int k = 0; k < 8; ++k) acc[k] += x[k];
                if (r < r1) *reinterpret_cast<uint4*>(dqkv + (size_t)r * 3 * D + c8 * 8) = f_to_h8(x);
            }
        }
    }
    if (qpart) fold_column_sums(acc, qpart + (size_t)blockIdx.y * D, c8, col_ok, red);
}

// dbias[off_w + c] += sum_b part[w][b][c] for w = 0 (q block, off 0) and, with
// gridDim.y == 2, w = 1 (v block, off 2D): 32 columns per CTA (one per lane),
// the 32 warps split the partial rows with four loads in flight, then fold in
// shared memory; a fixed summation order, so the bias gradients are
// deterministic.
__global__ void __launch_bounds__(1024) attn_bias_reduce_kernel(float* __restrict__ dbias,
                                                                const float* __restrict__ part, int nblk, int D) {
    grid_dependency_sync();
    __shared__ float s[32][33];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    const int w = blockIdx.y;
    const float* pw = part + (size_t)w * nblk * D;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (c < D) {
        int b = warp;
        for (; b + 96 < nblk; b += 128) {
#pragma unroll
            for (int u = 0; u < 4; ++u) acc[u] += __ldg(pw + (size_t)(b + 32 * u) * D + c);
        }
        for (; b < nblk; b += 32) acc[0] += __ldg(pw + (size_t)b * D + c);
    }
    s[warp][lane] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    __syncthreads();
    if (warp == 0 && c < D) {
        float t = 0.0f;
#pragma unroll 8
        for (int k = 0; k < 32; ++k) t += s[k][lane];
        dbias[(w ? 2 * D : 0) + c] += t;
    }
}

template <int HD>
int fwd(rbk_ctx* ctx, void* o, float* lse, const void* qkv, int B, int S, int H, float scale, cudaStream_t st) {
    constexpr int SMEM = 5 * BLK * HD * 2;
    static int set_dev = -1;
    if (set_dev != ctx->device) {
        RBK_CUDA(cudaFuncSetAttribute(flash_fwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        set_dev = ctx->device;
    }
    dim3 grid(S / BLK, B * H);
    flash_fwd_kernel<HD><<<grid, 128, SMEM, st>>>((half*)o, lse, (const half*)qkv, S, H, scale * kLog2e);
    RBK_LAUNCHED("flash_fwd_kernel");
    return RBK_OK;
}

template <int HD>
int bwd(rbk_ctx* ctx, void* dqkv, float* dbias, const void* qkv, const void* o, const void* dout, const float* lse,
        int B, int S, int H, float scale, bool tc, cudaStream_t st) {
    const int D = H * HD;
    const size_t BS = (size_t)B * S;
    const size_t dot_bytes = ((sizeof(float) * BS * H) + 255) & ~size_t(255);
    // Row-block layout of the pre / post passes: TX threads of 8 columns (a
    // warp multiple, at most 256, further column blocks beyond), TY row teams
    // (TX * TY <= 512), about two CTAs per SM, each over one contiguous row block.
    const int c8s = D / 8;
    const int TX = c8s >= 256 ? 256 : (c8s + 31) / 32 * 32;
    const int TY = 512 / TX;
    const int col_blocks = (c8s + TX - 1) / TX;
    int nrb = (2 * ctx->num_sms + col_blocks - 1) / col_blocks;
    if (nrb > (int)BS) nrb = (int)BS;
    const int rows_per_block = (int)((BS + nrb - 1) / nrb);
    nrb = (int)((BS + rows_per_block - 1) / rows_per_block);
    const size_t dq_bytes = (sizeof(float) * BS * D + 255) & ~size_t(255);
    const size_t part_bytes = sizeof(float) * (size_t)nrb * D;   // one [nrb, D] block per bias part
    const bool det = tc && ctx->deterministic;
    const int nsem = det ? (int)((size_t)B * H * (S / 64)) : 0;
    const size_t sem_bytes = ((sizeof(int) * (size_t)nsem) + 255) & ~size_t(255);
    void* ws;
    RBK_TRY(ctx_scratch(ctx, 2 * dot_bytes + dq_bytes + 2 * part_bytes + sem_bytes, &ws));
    int* sem = det ? (int*)((char*)ws + 2 * dot_bytes + dq_bytes + 2 * part_bytes) : nullptr;
    float* Dot = (float*)ws;
    float* NL2 = (float*)((char*)ws + dot_bytes);
    float* dq_acc = (float*)((char*)ws + 2 * dot_bytes);
    float* qpart = (float*)((char*)ws + 2 * dot_bytes + dq_bytes);
    float* vpart = (float*)((char*)qpart + part_bytes);
    // the tcgen05 main pass writes no bias terms: the v block comes from dO's column sums
    const bool vsum = dbias && tc;
    const dim3 rgrid(col_blocks, nrb), rblock(TX, TY);
    RBK_CUDA(launch_pdl(flash_bwd_pre_kernel<HD>, rgrid, rblock, 0, st, Dot, dq_acc, tc ? NL2 : nullptr,
                        vsum ? vpart : nullptr, lse, (const half*)o, (const half*)dout, (int)BS, S, H,
                        rows_per_block, sem, nsem));
    RBK_LAUNCHED("flash_bwd_pre_kernel");
    if (tc) {
        RBK_TRY(attn_bwd_tc(ctx, dqkv, dq_acc, qkv, dout, NL2, Dot, B, S, H, HD, scale, st, sem));
    } else {
        constexpr int SMEM = 6 * BLK * HD * 2 + BLK * BLK * 2 + 4 * BLK * 4;
        static int set_dev = -1;
        if (set_dev != ctx->device) {
            RBK_CUDA(cudaFuncSetAttribute(flash_bwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
            set_dev = ctx->device;
        }
        dim3 grid(S / BLK, B * H);
        flash_bwd_kernel<HD><<<grid, 128, SMEM, st>>>((half*)dqkv, dq_acc, dbias, (const half*)qkv,
                                                      (const half*)dout, lse, Dot, S, H, scale, scale * kLog2e);
        RBK_LAUNCHED("flash_bwd_kernel");
    }
    RBK_CUDA(launch_pdl(flash_bwd_post_kernel, rgrid, rblock, 0, st, (half*)dqkv, dbias ? qpart : nullptr,
                        (const float*)dq_acc, (int)BS, D, rows_per_block));
    RBK_LAUNCHED("flash_bwd_post_kernel");
    if (dbias) {
        RBK_CUDA(launch_pdl(attn_bias_reduce_kernel, dim3((D + 31) / 32, vsum ? 2 : 1), dim3(1024), 0, st, dbias,
                            (const float*)qpart, nrb, D));
        RBK_LAUNCHED("attn_bias_reduce_kernel");
    }
    return RBK_OK;
}

}  // namespace attn

// tcgen05 forward for d_head 64 / 128, S % 64 == 0 (attn_tc.cu).
int attn_fwd_tc(rbk_ctx* ctx, void* o, float* lse, const void* qkv, int B, int S, int H, int dh, float scale,
                cudaStream_t st);

}  // namespace rbk

using namespace rbk;

// RBK_ATTN_LEGACY=1 forces the mma.sync kernels for every shape (A/B comparisons).
static bool attn_legacy() {
    static const bool legacy = [] {
        const char* e = getenv("RBK_ATTN_LEGACY");
        return e && e[0] == '1';
    }();
    return legacy;
}

extern "C" {

int rbk_attn_fwd(rbk_ctx* ctx, void* o, float* lse, const void* qkv, int B, int S, int H, int dh, float scale,
                 void* stream) {
    RBK_REQUIRE(ctx && o && lse && qkv, "rbk_attn_fwd: null pointer");
    RBK_REQUIRE(B > 0 && H > 0 && S > 0 && S % 64 == 0, "rbk_attn_fwd: need S %% 64 == 0 (S=%d)", S);
    RBK_REQUIRE(dh == 64 || dh == 128, "rbk_attn_fwd: d_head must be 64 or 128 (got %d)", dh);
    RBK_REQUIRE(aligned16(o) && aligned16(qkv), "rbk_attn_fwd: 16-byte alignment");
    cudaStream_t st = as_stream(stream);
    // causal: QK^T and PV over S(S+1)/2 score entries per (b, h)
    ProfScope prof(ctx, st, kCatAttnFwd, 4.0 * B * H * ((double)S * (S + 1) / 2.0) * dh);
    // tcgen05 kernel (attn_tc.cu); the mma.sync kernels only under RBK_ATTN_LEGACY=1
    if (!attn_legacy()) return attn_fwd_tc(ctx, o, lse, qkv, B, S, H, dh, scale, st);
    return dh == 64 ? attn::fwd<64>(ctx, o, lse, qkv, B, S, H, scale, st)
                    : attn::fwd<128>(ctx, o, lse, qkv, B, S, H, scale, st);
}

int rbk_attn_bwd(rbk_ctx* ctx, void* dqkv, float* dbias_qkv, const void* qkv, const void* o, const void* dout,
                 const float* lse, int B, int S, int H, int dh, float scale, void* stream) {
    RBK_REQUIRE(ctx && dqkv && qkv && o && dout && lse, "rbk_attn_bwd: null pointer");
    RBK_REQUIRE(B > 0 && H > 0 && S > 0 && S % 64 == 0, "rbk_attn_bwd: need S %% 64 == 0 (S=%d)", S);
    RBK_REQUIRE(dh == 64 || dh == 128, "rbk_attn_bwd: d_head must be 64 or 128 (got %d)", dh);
    RBK_REQUIRE(aligned16(dqkv) && aligned16(qkv) && aligned16(o) && aligned16(dout), "rbk_attn_bwd: 16-byte alignment");
    cudaStream_t st = as_stream(stream);
    // algorithmic: dV, dP, dQ, dK products over the causal triangle (score recompute excluded)
    ProfScope prof(ctx, st, kCatAttnBwd, 8.0 * B * H * ((double)S * (S + 1) / 2.0) * dh);
    const bool tc = !attn_legacy();
    return dh == 64 ? attn::bwd<64>(ctx, dqkv, dbias_qkv, qkv, o, dout, lse, B, S, H, scale, tc, st)
                    : attn::bwd<128>(ctx, dqkv, dbias_qkv, qkv, o, dout, lse, B, S, H, scale, tc, st);
}

}  // extern "C"
