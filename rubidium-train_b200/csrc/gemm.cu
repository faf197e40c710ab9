// gemm.cu — FP16 x FP16 -> FP32 GEMM on the 5th-generation tensor cores.
//
// C[M,N] = op(A)[M,K] . op(B)[N,K]^T with fused epilogues; every dense
// contraction of the model (forward linears, dgrad, wgrad, LM head) runs here.
// It replaces the reference's cuBLAS/cuBLASLt wrappers and naive fused kernels
// (src/cuda_kernels.cu:596-665, 670-784, 1031-1045).
//
// Design (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: 128B-swizzled tiles of A (128 x 64) and B
//               (BN x 64) into a STAGES-deep shared-memory ring (mbarriers with
//               complete_tx).  K-major operands are one box per tile; MN-major
//               operands (the transposed reads of dgrad/wgrad) are 64-wide
//               boxes stacked at the descriptor's leading-byte offset.
//   warp 1      MMA issuer: tcgen05.mma.cta_group::1.kind::f16, M=128, N=BN,
//               K=16 per instruction, FP32 accumulator in TMEM, double-buffered
//               so the epilogue of tile i overlaps the MMAs of tile i+1.
//               tcgen05.commit releases smem stages and publishes accumulators.
//   warps 2..5  epilogue: tcgen05.ld 32x32b (one TMEM lane quarter per warp,
//               one output row per thread), fused bias / residual / GELU /
//               GELU' / FP32 accumulation, direct 16-byte global stores.
// Bias gradients (row sums of A over K when A = dY^T): in this 1-CTA kernel one
// extra N=16 MMA per k-step against a constant ones tile, issued by the n=0
// tiles; in the CTA-pair kernel below an extra warp sums A from shared memory.
// Every mbarrier wait is bounded (globaltimer); on expiry the kernel records
// RBK_ERR_TIMEOUT, drains, frees TMEM and returns.
// No cluster multicast is used anywhere.
#include <type_traits>

#include "tc.cuh"

namespace rbk {
namespace gemm {

constexpr int BM = 128, BK = 64, UMMA_K = 16;
constexpr int kEpiWarps = 8;                  // two warps per TMEM lane quarter, split by columns
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kStageRow = 80;                 // epilogue staging tile: 32 rows x (64 B + 16 B pad)
constexpr int kStageBytes = 32 * kStageRow;

// GELU with the hardware tanh (tanh.approx.f32, ~2^-11 relative error: the
// size of the FP16 rounding that follows).  GPT-2 tanh form, as the oracle.
__device__ __forceinline__ float tanh_fast(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float gelu_fast(float x) {
    const float c = 0.7978845608028654f, a = 0.044715f;
    return 0.5f * x * (1.0f + tanh_fast(c * (x + a * x * x * x)));
}
__device__ __forceinline__ float gelu_grad_fast(float x) {
    const float c = 0.7978845608028654f, a = 0.044715f;
    const float t = tanh_fast(c * (x + a * x * x * x));
    return 0.5f * (1.0f + t) + 0.5f * x * (1.0f - t * t) * c * (1.0f + 3.0f * a * x * x);
}
// Two lanes at once with packed FP32 pairs (sm_100 fma/mul.rn.f32x2); the same
// formulas: gelu = x (0.5 + 0.5 t), gelu' = 0.5 (1 + t) + 0.5 x (1 - t^2) c (1 + 3 a x^2),
// t = tanh(c x (1 + a x^2)).
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
    return ((uint64_t)__float_as_uint(b) << 32) | __float_as_uint(a);
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& a, float& b) {
    a = __uint_as_float((uint32_t)v);
    b = __uint_as_float((uint32_t)(v >> 32));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ void gelu2(float& x0, float& x1) {
    const uint64_t c2 = f2pack(0.7978845608028654f, 0.7978845608028654f), a2 = f2pack(0.044715f, 0.044715f);
    const uint64_t one2 = f2pack(1.0f, 1.0f), half2 = f2pack(0.5f, 0.5f);
    const uint64_t x = f2pack(x0, x1);
    const uint64_t u = mul2(mul2(x, c2), fma2(mul2(x, x), a2, one2));   // c x (1 + a x^2)
    float u0, u1;
    f2unpack(u, u0, u1);
    const uint64_t t = f2pack(tanh_fast(u0), tanh_fast(u1));
    f2unpack(mul2(x, fma2(t, half2, half2)), x0, x1);
}
// (g0, g1) *= gelu'(x0, x1)
__device__ __forceinline__ void gelu_grad2(float& g0, float& g1, float x0, float x1) {
    const float c = 0.7978845608028654f, a = 0.044715f;
    const uint64_t c2 = f2pack(c, c), a2 = f2pack(a, a), a3c = f2pack(3.0f * a, 3.0f * a);
    const uint64_t one2 = f2pack(1.0f, 1.0f), half2 = f2pack(0.5f, 0.5f), hc2 = f2pack(0.5f * c, 0.5f * c);
    const uint64_t mone2 = f2pack(-1.0f, -1.0f);
    const uint64_t x = f2pack(x0, x1), xx = mul2(x, x);
    const uint64_t u = mul2(mul2(x, c2), fma2(xx, a2, one2));
    float u0, u1;
    f2unpack(u, u0, u1);
    const uint64_t t = f2pack(tanh_fast(u0), tanh_fast(u1));
    const uint64_t omt = fma2(mul2(t, t), mone2, one2);                 // 1 - t^2
    const uint64_t r = mul2(mul2(x, hc2), mul2(omt, fma2(xx, a3c, one2)));   // 0.5 c x (1 - t^2)(1 + 3 a x^2)
    const uint64_t d = fma2(t, half2, fma2(one2, half2, r));              // 0.5 + 0.5 t + r
    f2unpack(mul2(f2pack(g0, g1), d), g0, g1);
}

template <int BN>
struct Cfg {
    static constexpr int STAGES = BN == 256 ? 4 : BN == 192 ? 5 : 6;
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int ONES_BYTES = 16 * BK * 2;
    static constexpr int BAR_BYTES = 256;
    static constexpr int EPI_BYTES = kEpiWarps * kStageBytes;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + ONES_BYTES + EPI_BYTES + BAR_BYTES;
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr int ACC2_COL = 2 * BN;   // ones-MMA accumulators (BN <= 192 only)
    static constexpr bool ROWSUM_OK = 2 * BN + 32 <= (int)TMEM_COLS;
};

struct Params {
    int M, N, K;
    int m_blocks, n_blocks, k_blocks, splits, kb_per_split, units;
    int a_mn, b_mn;
    void* C;
    int ldc;
    const half* bias;
    const half* aux;
    int ld_aux;
    half* aux_out;
    float* dbias_rows;
    float alpha;
    int* err;
    // FP32 accumulation (ACC_F32) without atomics where possible: the units of split 0 own C and
    // add their tile with plain loads and stores when no other unit writes it concurrently (one
    // split, or deterministic mode); in deterministic mode the units of split s >= 1 store their
    // partial tile (alpha applied) into plane s - 1, and splitk_reduce_kernel adds the planes to C
    // in split order.  Otherwise (several splits, atomic mode) every unit reduce-adds into C.
    float* part;        // [splits - 1][M][ldp], or nullptr (atomic mode)
    float* part_rows;   // [splits - 1][M] row-sum partials (dbias_rows)
    int ldp;            // row pitch of a plane (N rounded up to 4)
    int c_zero;         // ACC_F32 into a C known to hold zeros: the owner stores without reading C
};

// How an ACC_F32 unit of split `split` writes its tile.  kAccStore: the owner of a tile whose C
// holds zeros stores its values (C + acc = acc) instead of reading C first.
enum AccMode { kAccAtomic = 0, kAccOwner = 1, kAccPlane = 2, kAccStore = 3 };
__device__ __forceinline__ int acc_mode(const Params& p, int split) {
    if (split == 0 && (p.splits == 1 || p.part)) return p.c_zero ? kAccStore : kAccOwner;
    return p.part ? kAccPlane : kAccAtomic;
}

// PTX helpers (mbarriers, TMA, tcgen05, descriptors) come from tc.cuh.
using namespace tc;

__device__ __forceinline__ void decode_unit(const Params& p, int u, int& m_blk, int& n_blk, int& kb0, int& kb1) {
    const int split = u % p.splits;
    const int tile = u / p.splits;
    constexpr int GM = 8;
    const int group_size = GM * p.n_blocks;
    const int group = tile / group_size;
    const int first_m = group * GM;
    const int gm = min(GM, p.m_blocks - first_m);
    const int in_group = tile - group * group_size;
    m_blk = first_m + in_group % gm;
    n_blk = in_group / gm;
    kb0 = split * p.kb_per_split;
    kb1 = min(p.k_blocks, kb0 + p.kb_per_split);
}

// ------------------------------------------------------------- epilogue ----
// Every epilogue warp owns a 32-row x 32-column chunk at a time (thread =
// row, as tcgen05.ld 32x32b delivers it).  Global traffic goes through a
// private shared tile (32 rows x 80 B: 64 B of data + 16 B pad, so each
// 8-thread phase of a 16-byte access hits distinct banks) and is issued
// row-segment-wise: lane -> (row lane/4 + 8i, 16-byte piece lane%4), i.e. each
// instruction covers 8 full 64-byte row segments instead of 32 scattered
// 16-byte pieces.
// Coalesced loads of a 32 x 32 half tile (row pitch ld) into registers: lane
// holds pieces (row lane/4 + 8i, 16-byte piece lane%4).  Issued one chunk
// ahead so the HBM latency overlaps the previous chunk (or the MMAs).
__device__ __forceinline__ void prefetch_h(uint4* pf, const half* g, int ld, int m0, int n, const Params& p,
                                           int lane) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int rr = i * 8 + (lane >> 2), pc = lane & 3;
        const int m = m0 + rr, col = n + 8 * pc;
        uint4 u = make_uint4(0, 0, 0, 0);
        if (m < p.M && col < p.N) {
            const half* src = g + (size_t)m * ld + col;
            if (col + 8 <= p.N) {
                u = __ldg(reinterpret_cast<const uint4*>(src));
            } else {
                half h[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) h[e] = col + e < p.N ? src[e] : __float2half(0.0f);
                u = *reinterpret_cast<uint4*>(h);
            }
        }
        pf[i] = u;
    }
}
__device__ __forceinline__ void stage_in_h(uint8_t* st, const uint4* pf, int lane) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
        *reinterpret_cast<uint4*>(st + (i * 8 + (lane >> 2)) * kStageRow + (lane & 3) * 16) = pf[i];
}
// Coalesced stage -> global for a 32 x 32 half tile.
__device__ __forceinline__ void stage_out_h(const uint8_t* st, half* g, int ld, int m0, int n, const Params& p,
                                            int lane) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int rr = i * 8 + (lane >> 2), pc = lane & 3;
        const int m = m0 + rr, col = n + 8 * pc;
        if (m >= p.M || col >= p.N) continue;
        const uint4 u = *reinterpret_cast<const uint4*>(st + rr * kStageRow + pc * 16);
        half* dst = g + (size_t)m * ld + col;
        if (col + 8 <= p.N) {
            *reinterpret_cast<uint4*>(dst) = u;
        } else {
            const half* h = reinterpret_cast<const half*>(&u);
#pragma unroll
            for (int e = 0; e < 8; ++e)
                if (col + e < p.N) dst[e] = h[e];
        }
    }
}
// Own row (thread = row) <-> stage, 32 halves as 4 x 16 B.
__device__ __forceinline__ void row_to_stage_h(uint8_t* st, int lane, const float* v) {
#pragma unroll
    for (int k = 0; k < 4; ++k) *reinterpret_cast<uint4*>(st + lane * kStageRow + k * 16) = f_to_h8(v + 8 * k);
}
__device__ __forceinline__ void row_from_stage_h(const uint8_t* st, int lane, float* v) {
#pragma unroll
    for (int k = 0; k < 4; ++k) h8_to_f(*reinterpret_cast<const uint4*>(st + lane * kStageRow + k * 16), v + 8 * k);
}

// r: 32 FP32 accumulators of row m0 + lane, columns n .. n+31.
// pf: this chunk's aux pieces (prefetch_h), used when p.aux is set.
template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const Params& p, int m0, int n, const uint32_t* r, uint8_t* st,
                                               int lane, const uint4* pf, int mode = kAccAtomic,
                                               float* plane = nullptr) {
    if (n >= p.N || m0 >= p.M) return;                     // warp-uniform: nothing of this chunk is in C
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);

    if constexpr (EPI == RBK_EPI_ACC_F32 || EPI == RBK_EPI_STORE_F32) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] *= p.alpha;
        float* C = reinterpret_cast<float*>(p.C);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {             // 16 FP32 columns (64 B per row) at a time
#pragma unroll
            for (int k = 0; k < 4; ++k)
                *reinterpret_cast<float4*>(st + lane * kStageRow + k * 16) =
                    make_float4(v[16 * hh + 4 * k], v[16 * hh + 4 * k + 1], v[16 * hh + 4 * k + 2],
                                v[16 * hh + 4 * k + 3]);
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int rr = i * 8 + (lane >> 2), pc = lane & 3;
                const int m = m0 + rr, col = n + 16 * hh + 4 * pc;
                if (m < p.M && col < p.N) {
                    const float4 f = *reinterpret_cast<const float4*>(st + rr * kStageRow + pc * 16);
                    const bool pl = EPI == RBK_EPI_ACC_F32 && mode == kAccPlane;
                    float* dst = pl ? plane + (size_t)m * p.ldp + col : C + (size_t)m * p.ldc + col;
                    if (col + 4 <= p.N) {
                        if (EPI == RBK_EPI_ACC_F32 && mode == kAccAtomic) {
                            red_add_v4(dst, f.x, f.y, f.z, f.w);
                        } else if (EPI == RBK_EPI_ACC_F32 && mode == kAccOwner) {
                            float4 o = *reinterpret_cast<const float4*>(dst);
                            o.x += f.x; o.y += f.y; o.z += f.z; o.w += f.w;
                            *reinterpret_cast<float4*>(dst) = o;
                        } else {
                            *reinterpret_cast<float4*>(dst) = f;
                        }
                    } else {
                        const float fv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            if (col + e < p.N) {
                                if (EPI == RBK_EPI_ACC_F32 && mode == kAccAtomic) atomicAdd(dst + e, fv[e]);
                                else if (EPI == RBK_EPI_ACC_F32 && mode == kAccOwner) dst[e] += fv[e];
                                else dst[e] = fv[e];
                            }
                        }
                    }
                }
            }
            __syncwarp();
        }
        return;
    } else {
        const int lda = p.ld_aux ? p.ld_aux : p.ldc;
        if constexpr (EPI == RBK_EPI_STORE_F16) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] *= p.alpha;
        }
        if (p.bias && EPI != RBK_EPI_GELU_BWD) {          // one 64-byte bias row, broadcast to all lanes
            if (n + 32 <= p.N) {
#pragma unroll
                for (int j = 0; j < 32; j += 8) {
                    float b[8];
                    h8_to_f(__ldg(reinterpret_cast<const uint4*>(p.bias + n + j)), b);
#pragma unroll
                    for (int q = 0; q < 8; ++q) v[j + q] += b[q];
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (n + j < p.N) v[j] += __half2float(p.bias[n + j]);
            }
        }
        if (p.aux) {                                       // residual or GELU pre-activation
            stage_in_h(st, pf, lane);
            __syncwarp();
            float b[32];
            row_from_stage_h(st, lane, b);
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                if constexpr (EPI == RBK_EPI_GELU_BWD) v[j] *= gelu_grad_fast(b[j]);
                else v[j] += b[j];
            }
        }
        row_to_stage_h(st, lane, v);
        __syncwarp();
        if (p.C) stage_out_h(st, reinterpret_cast<half*>(p.C), p.ldc, m0, n, p, lane);
        __syncwarp();
        if constexpr (EPI == RBK_EPI_BIAS_GELU) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = gelu_fast(v[j]);
            row_to_stage_h(st, lane, v);
            __syncwarp();
            stage_out_h(st, p.aux_out, lda, m0, n, p, lane);
            __syncwarp();
        }
    }
}

// Deterministic split K: C[m, n] += part[0][m][n] + part[1][m][n] + ... in plane (split) order,
// after split 0 has added its own tile (and dbias_rows[m] += the row-sum planes), one thread per
// 4 columns, four planes' loads in flight.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(float* __restrict__ C, int ldc, const float* __restrict__ part,
                                                            int M, int N, int ldp, int splits, float* __restrict__ dbias,
                                                            const float* __restrict__ part_rows) {
    grid_dependency_sync();
    const size_t plane = (size_t)M * ldp;
    const int q4 = (N + 3) >> 2;
    const size_t total = (size_t)M * q4;
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += stride) {
        const int m = (int)(i / q4), c = (int)(i - (size_t)m * q4) * 4;
        const float* src = part + (size_t)m * ldp + c;
        float* dst = C + (size_t)m * ldc + c;
        if (c + 4 <= N) {
            float4 a = *reinterpret_cast<const float4*>(dst);
            int sp = 0;
            for (; sp + 4 <= splits; sp += 4) {                 // four planes' loads in flight at once
                float4 b[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) b[j] = __ldcs(reinterpret_cast<const float4*>(src + (sp + j) * plane));
#pragma unroll
                for (int j = 0; j < 4; ++j) { a.x += b[j].x; a.y += b[j].y; a.z += b[j].z; a.w += b[j].w; }
            }
            for (; sp < splits; ++sp) {
                const float4 b = __ldcs(reinterpret_cast<const float4*>(src + sp * plane));
                a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
            }
            *reinterpret_cast<float4*>(dst) = a;
        } else {
            for (int e = 0; c + e < N; ++e) {
                float a = dst[e];
                for (int sp = 0; sp < splits; ++sp) a += src[sp * plane + e];
                dst[e] = a;
            }
        }
    }
    if (dbias) {
        for (size_t m = blockIdx.x * (size_t)blockDim.x + threadIdx.x; m < (size_t)M; m += stride) {
            float a = dbias[m];
            for (int sp = 0; sp < splits; ++sp) a += part_rows[(size_t)sp * M + m];
            dbias[m] = a;
        }
    }
}

// ----------------------------------------------------------------- kernel ----
template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                           const __grid_constant__ CUtensorMap tmB, const Params p) {
    using C = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = su32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw);
    const uint32_t sA0 = base;                                       // stage s: A at s*STAGE_BYTES
    const uint32_t ones = base + C::STAGES * C::STAGE_BYTES;          // 2 KB of fp16 ones
    const uint32_t epi_stage = ones + C::ONES_BYTES;                 // kEpiWarps x kStageBytes
    const uint32_t bars = epi_stage + C::EPI_BYTES;
    uint8_t* gbars = gbase + (bars - base);
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (C::STAGES + s); };
    auto tfull_bar = [&](int b) { return bars + 8u * (2 * C::STAGES + b); };
    auto tempty_bar = [&](int b) { return bars + 8u * (2 * C::STAGES + 2 + b); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbars + 8 * (2 * C::STAGES + 4));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gbars + 8 * (2 * C::STAGES + 4) + 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // ones tile (for the bias-gradient MMA) and barrier init
    {
        uint32_t* o = reinterpret_cast<uint32_t*>(gbase + (ones - base));
        for (int i = threadIdx.x; i < C::ONES_BYTES / 4; i += blockDim.x) o[i] = 0x3C003C00u;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), kEpiWarps);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0 && lane == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(C::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_dependency_sync();

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x) {
                int mb, nb, kb0, kb1;
                decode_unit(p, u, mb, nb, kb0, kb1);
                const int m0 = mb * BM, n0 = nb * BN;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag)) break;
                    const uint32_t fb = full_bar(stage);
                    mbar_expect_tx(fb, C::STAGE_BYTES);
                    const uint32_t sa = sA0 + stage * C::STAGE_BYTES;
                    const uint32_t sb = sa + C::A_BYTES;
                    const int k0 = kb * BK;
                    if (!p.a_mn) {
                        tma_load_2d(sa, &tmA, fb, k0, m0);
                    } else {
                        tma_load_2d(sa, &tmA, fb, m0, k0);
                        tma_load_2d(sa + 8192, &tmA, fb, m0 + 64, k0);
                    }
                    if (!p.b_mn) {
                        tma_load_2d(sb, &tmB, fb, k0, n0);
                    } else {
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + 8192 * j, &tmB, fb, n0 + 64 * j, k0);
                    }
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer --------------------------
        if (lane == 0) {
            const uint32_t idesc = idesc_f16(BN, p.a_mn, p.b_mn);
            const uint32_t idesc1 = idesc_f16(16, p.a_mn, 0);
            const uint32_t a_lbo = p.a_mn ? 8192u : 16u, b_lbo = p.b_mn ? 8192u : 16u;
            const uint32_t a_kstep = p.a_mn ? 2048u : 32u, b_kstep = p.b_mn ? 2048u : 32u;
            int stage = 0, buf = 0;
            uint32_t phase = 0, bphase = 0;
            for (int u = blockIdx.x; u < p.units && !*abort_flag; u += gridDim.x) {
                int mb, nb, kb0, kb1;
                decode_unit(p, u, mb, nb, kb0, kb1);
                const bool rowsum = EPI == RBK_EPI_ACC_F32 && C::ROWSUM_OK && p.dbias_rows && nb == 0;
                if (!mbar_wait(tempty_bar(buf), bphase ^ 1, abort_flag)) break;
                fence_after();
                const uint32_t dacc = tmem + buf * BN;
                const uint32_t dacc2 = tmem + C::ACC2_COL + buf * 16;
                // two versions of the k-loop: no per-MMA branch in the issuing thread
                auto mainloop = [&](auto with_rows) -> bool {
                    constexpr bool kRows = decltype(with_rows)::value;
                    for (int kb = kb0; kb < kb1; ++kb) {
                        if (!mbar_wait(full_bar(stage), phase, abort_flag)) return false;
                        fence_after();
                        const uint32_t sa = sA0 + stage * C::STAGE_BYTES;
                        const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
                        for (int k = 0; k < BK / UMMA_K; ++k) {
                            const uint64_t ad = sdesc(sa + k * a_kstep, a_lbo, 1024);
                            const uint64_t bd = sdesc(sb + k * b_kstep, b_lbo, 1024);
                            const uint32_t acc = (kb > kb0 || k > 0) ? 1u : 0u;
                            mma_f16(dacc, ad, bd, idesc, acc);
                            if constexpr (kRows) mma_f16(dacc2, ad, sdesc(ones + k * 32, 16, 1024), idesc1, acc);
                        }
                        mma_commit(empty_bar(stage));
                        if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
                    }
                    return true;
                };
                bool ok;
                if constexpr (EPI == RBK_EPI_ACC_F32) ok = rowsum ? mainloop(std::true_type{}) : mainloop(std::false_type{});
                else ok = mainloop(std::false_type{});
                if (!ok) break;
                mma_commit(tfull_bar(buf));
                if (++buf == 2) { buf = 0; bphase ^= 1; }
            }
        }
    } else {
        // ------------------------------ epilogue ----------------------------
        const int q = warp & 3;                 // TMEM lane quarter of this warp
        const int half_id = (warp - 2) / 4;     // which half of the tile's columns
        constexpr int kChunks = BN / 32;
        const int c0 = half_id * (kChunks / 2), c1 = half_id ? kChunks : kChunks / 2;
        const int row = q * 32 + lane;
        uint8_t* my_stage = gbase + (epi_stage - base) + (warp - 2) * kStageBytes;
        int buf = 0;
        uint32_t bphase = 0;
        for (int u = blockIdx.x; u < p.units; u += gridDim.x) {
            int mb, nb, kb0, kb1;
            decode_unit(p, u, mb, nb, kb0, kb1);
            const int m0 = mb * BM + q * 32;
            const int split = u % p.splits;
            const int mode = acc_mode(p, split);
            float* plane = mode == kAccPlane ? p.part + (size_t)(split - 1) * p.M * p.ldp : nullptr;
            // residual / pre-activation of the first chunk: fetched while the MMAs run
            constexpr bool kAux = EPI == RBK_EPI_STORE_F16 || EPI == RBK_EPI_BIAS_GELU || EPI == RBK_EPI_GELU_BWD;
            const int lda = p.ld_aux ? p.ld_aux : p.ldc;
            uint4 pf[4];
            if (kAux && p.aux) prefetch_h(pf, p.aux, lda, m0, nb * BN + c0 * 32, p, lane);
            if (!mbar_wait(tfull_bar(buf), bphase, abort_flag)) break;
            fence_after();
            const int m = mb * BM + row;
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + buf * BN;
#pragma unroll 1
            for (int c = c0; c < c1; ++c) {
                uint32_t r[32];
                tmem_ld32(tbase + c * 32, r);
                uint4 cur[4] = {pf[0], pf[1], pf[2], pf[3]};
                if (kAux && p.aux && c + 1 < c1) prefetch_h(pf, p.aux, lda, m0, nb * BN + (c + 1) * 32, p, lane);
                tmem_wait_ld();
                epilogue_chunk<EPI>(p, m0, nb * BN + c * 32, r, my_stage, lane, cur, mode, plane);
            }
            const bool rowsum_tile = EPI == RBK_EPI_ACC_F32 && C::ROWSUM_OK && p.dbias_rows && nb == 0;
            if (rowsum_tile && half_id == 0) {
                const uint32_t v = tmem_ld1(tmem + ((uint32_t)(q * 32) << 16) + C::ACC2_COL + buf * 16);
                tmem_wait_ld();
                if (m < p.M) {
                    const float bv = p.alpha * __uint_as_float(v);
                    if (mode == kAccPlane) p.part_rows[(size_t)(split - 1) * p.M + m] = bv;
                    else if (mode == kAccOwner) p.dbias_rows[m] += bv;
                    else atomicAdd(p.dbias_rows + m, bv);
                }
            }
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(buf));
            if (++buf == 2) { buf = 0; bphase ^= 1; }
        }
    }

    fence_before();
    __syncthreads();
    fence_after();
    if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, RBK_ERR_TIMEOUT);
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
}

// ------------------------------------------------- TMA-store epilogue ----
// FP16 outputs of the CTA-pair kernel leave through a tensor store: the warp
// writes its 32 x 32 chunk into a 2 KB shared tile in the 64-byte swizzle
// (16-byte piece pc of row r at r * 64 + ((pc ^ ((r >> 1) & 3)) << 4), free of
// bank conflicts for a thread per row and for 2 rows x 4 pieces), and one lane
// issues cp.async.bulk.tensor; the map's extents clip rows >= M and columns >= N.
// Each warp owns two such tiles (4 KB).
__device__ __forceinline__ int swoff(int r, int pc) { return r * 64 + ((pc ^ ((r >> 1) & 3)) << 4); }
__device__ __forceinline__ void row_to_sw(uint8_t* st, int lane, const float* v) {
#pragma unroll
    for (int k = 0; k < 4; ++k) *reinterpret_cast<uint4*>(st + swoff(lane, k)) = f_to_h8(v + 8 * k);
}
__device__ __forceinline__ void stage_in_sw(uint8_t* st, const uint4* pf, int lane) {
#pragma unroll
    for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(st + swoff(i * 8 + (lane >> 2), lane & 3)) = pf[i];
}
__device__ __forceinline__ void row_from_sw(const uint8_t* st, int lane, float* v) {
#pragma unroll
    for (int k = 0; k < 4; ++k) h8_to_f(*reinterpret_cast<const uint4*>(st + swoff(lane, k)), v + 8 * k);
}
constexpr int kTmaStageBytes = 4096;            // per epilogue warp: two 2 KB tiles

// FP16 epilogues (STORE_F16, BIAS_GELU, GELU_BWD) of one 32 x 32 chunk through
// tensor stores.  st / st_s: the warp's two tiles (generic / shared address);
// sc: the warp's chunk counter (single-output chunks alternate tiles).
template <int EPI>
__device__ __forceinline__ void epilogue_chunk_tma(const Params& p, int m0, int n, const uint32_t* r, uint8_t* st,
                                                   uint32_t st_s, int lane, const uint4* pf, const CUtensorMap* tmC,
                                                   const CUtensorMap* tmX, int& sc) {
    if (n >= p.N || m0 >= p.M) return;                     // warp-uniform: nothing of this chunk is in C
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    if constexpr (EPI == RBK_EPI_STORE_F16) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] *= p.alpha;
    }
    if (p.bias && EPI != RBK_EPI_GELU_BWD) {
        if (n + 32 <= p.N) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
                float b[8];
                h8_to_f(__ldg(reinterpret_cast<const uint4*>(p.bias + n + j)), b);
#pragma unroll
                for (int q = 0; q < 8; ++q) v[j + q] += b[q];
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (n + j < p.N) v[j] += __half2float(p.bias[n + j]);
        }
    }
    constexpr bool kTwo = EPI == RBK_EPI_BIAS_GELU;
    const int t = kTwo ? 0 : (sc & 1);
    uint8_t* tile = st + t * 2048;
    if (lane == 0) {                                       // the tile's previous tensor store has read it
        if (kTwo) bulk_wait_read0();
        else bulk_wait_read1();
    }
    __syncwarp();
    if (p.aux) {                                           // residual or GELU pre-activation
        stage_in_sw(tile, pf, lane);
        __syncwarp();
        float b[32];
        row_from_sw(tile, lane, b);
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
            if constexpr (EPI == RBK_EPI_GELU_BWD) {
                gelu_grad2(v[j], v[j + 1], b[j], b[j + 1]);
            } else {
                v[j] += b[j];
                v[j + 1] += b[j + 1];
            }
        }
    }
    const bool store_c = !kTwo || p.C != nullptr;       // BIAS_GELU may store the activation only
    if (store_c) row_to_sw(tile, lane, v);
    if constexpr (kTwo) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) gelu2(v[j], v[j + 1]);
        row_to_sw(st + 2048, lane, v);
    }
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
        if (store_c) tma_store_2d(tmC, st_s + t * 2048, n, m0);
        if constexpr (kTwo) tma_store_2d(tmX, st_s + 2048, n, m0);
        bulk_commit();
    }
    ++sc;
}

// FP32 epilogues (ACC_F32, STORE_F32) of one 32 x 32 chunk through bulk tensor operations: two
// 32-row x 16-column halves (64-byte rows, the same 64-byte swizzle as the FP16 tiles) leave
// through the warp's 2 KB tile, each half as one tensor reduce-add into C (ACC_F32) or one tensor
// store (STORE_F32, and the split planes of deterministic mode: tmP, a 3-D map [splits][M][ldp]
// whose z coordinate is the split).  One bulk request per 2 KB instead of 128 per-lane vector
// reductions; the map's extents clip rows >= M and columns >= N.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* tm, uint32_t src, int x, int y, int z) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(tm),
                 "r"(src), "r"(x), "r"(y), "r"(z)
                 : "memory");
}
// Row m0 + lane of C, columns n .. n + 31 (the owner's read of the values it adds to), 16 B at a
// time; rows >= M and columns >= N read as zero.
__device__ __forceinline__ void load_c_row(float4* cv, const Params& p, int m0, int n, int lane) {
    const int m = m0 + lane;
    const float* src = reinterpret_cast<const float*>(p.C) + (size_t)m * p.ldc + n;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int col = n + 4 * k;
        cv[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (m < p.M && col < p.N) {
            if (col + 4 <= p.N) {
                cv[k] = __ldcg(reinterpret_cast<const float4*>(src + 4 * k));
            } else {
                float t[4] = {0.f, 0.f, 0.f, 0.f};
                for (int e = 0; col + e < p.N; ++e) t[e] = src[4 * k + e];
                cv[k] = make_float4(t[0], t[1], t[2], t[3]);
            }
        }
    }
}

template <int EPI>
__device__ __forceinline__ void epilogue_chunk_f32_tma(const Params& p, int m0, int n, const uint32_t* r,
                                                       uint8_t* st, uint32_t st_s, int lane, const CUtensorMap* tmC,
                                                       const CUtensorMap* tmP, int split, int mode, const float4* cv) {
    if (n >= p.N || m0 >= p.M) return;                     // warp-uniform: nothing of this chunk is in C
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {                       // half hh uses tile hh: one operation may stay in flight
        if (lane == 0) bulk_wait_read1();                  // the tile's previous bulk operation has read it
        __syncwarp();
        uint8_t* tile = st + hh * 2048;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int j = 16 * hh + 4 * k;
            float4 v = make_float4(__uint_as_float(r[j]) * p.alpha, __uint_as_float(r[j + 1]) * p.alpha,
                                   __uint_as_float(r[j + 2]) * p.alpha, __uint_as_float(r[j + 3]) * p.alpha);
            if (EPI == RBK_EPI_ACC_F32 && mode == kAccOwner) {
                const float4 c = cv[4 * hh + k];
                v.x += c.x; v.y += c.y; v.z += c.z; v.w += c.w;
            }
            *reinterpret_cast<float4*>(tile + swoff(lane, k)) = v;
        }
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
            const uint32_t ts = st_s + hh * 2048;
            if (EPI == RBK_EPI_ACC_F32 && mode == kAccPlane) tma_store_3d(tmP, ts, n + 16 * hh, m0, split - 1);
            else if (EPI == RBK_EPI_ACC_F32 && mode == kAccAtomic) tma_reduce_add_2d(tmC, ts, n + 16 * hh, m0);
            else tma_store_2d(tmC, ts, n + 16 * hh, m0);
            bulk_commit();
        }
    }
}

// ------------------------------------------------------------ CTA pairs ----
// The same GEMM on CTA pairs (a 2-CTA cluster per pair of SMs): a pair tile is
// 256 rows x 256 columns.  Each CTA stages its 128 rows of A and its 128
// columns of B per k-block (32 KB a stage instead of 48 KB for a 1-CTA
// 128 x 256 tile), and the even CTA issues tcgen05.mma.cta_group::2 with
// M = 256, N = 256, which reads A and B from both CTAs' shared memory and
// leaves each CTA's 128 accumulator rows in its own TMEM.  Per SM and k-step
// the tensor pipe then needs 8 KB of operands from shared memory and 8 KB
// written by TMA, against 12 + 12 KB on a 1-CTA N = 256 tile: the 1-CTA tile
// is bound by shared-memory bandwidth, the pair tile is not.
// Barriers: full[s] lives in the even CTA and counts the TMA bytes of both
// CTAs; empty[s] and tfull[b] exist in both CTAs and get one commit each from
// the MMA thread; tempty[b] lives in the even CTA and takes the arrivals of
// both CTAs' epilogue warps.  Bounded waits as in gemm_kernel.
constexpr int kPairStages = 6;
// Shared-memory loads and FP32 += FP16 pair additions for the row warp.
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ void add_f16x2(float& c0, float& c1, uint32_t a) {
    asm("{.reg .f16 al, ah;\n\t"
        "mov.b32 {al, ah}, %2;\n\t"
        "add.rn.f32.f16 %0, al, %0;\n\t"
        "add.rn.f32.f16 %1, ah, %1;}"
        : "+f"(c0), "+f"(c1)
        : "r"(a));
}

// Per-warp epilogue staging: two 2 KB tiles for the tensor stores / reduce-adds; the FP32
// epilogues run one operand stage fewer (their K = tokens mainloops are long).
constexpr int kRowWarps = 5;                    // ROW: row warp w owns operand stage w
template <int EPI, bool ROW>
struct PairEpi {
    static constexpr bool TMA = EPI == RBK_EPI_STORE_F16 || EPI == RBK_EPI_BIAS_GELU || EPI == RBK_EPI_GELU_BWD;
    static constexpr int STAGES = TMA ? kPairStages : kPairStages - 1;
    static constexpr int WARP_STAGE = kTmaStageBytes;
    static constexpr int PART_BYTES = ROW ? kRowWarps * BM * 4 : 0;     // per-warp row partials
    static constexpr int SMEM = 1024 + STAGES * (BM * BK * 2 + 128 * BK * 2) + kEpiWarps * WARP_STAGE +
                                PART_BYTES + 256;
    static constexpr int THREADS = kThreads + (ROW ? 32 * kRowWarps : 0);
};
// ROW: the ACC_F32 instance that also produces the row sums of A (the bias gradient of a weight
// gradient, A = dY^T, into dbias_rows).  One row warp per operand stage (kRowWarps per CTA)
// sums the CTA's 128 rows of A of the n = 0 tiles from shared memory after the MMAs have
// consumed a stage: for those tiles the MMA thread's commits go to a per-stage `consumed`
// barrier in each CTA, and the stage's row warp frees it for the producer; the other tiles free
// their stages directly.  At the end of an n = 0 tile the warps' partials are added in warp
// order (bounded mbarrier hand-off), so the result does not depend on timing.  The tensor pipe
// does no row-sum work and both TMEM accumulator buffers stay in use.
template <int EPI, bool ROW>
__global__ void __launch_bounds__(PairEpi<EPI, ROW>::THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmX,
                     const __grid_constant__ CUtensorMap tmP, const Params p) {
    constexpr int BN = 256, HALF_N = 128;
    constexpr int A_BYTES = BM * BK * 2, B_BYTES = HALF_N * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
    constexpr int STAGES = PairEpi<EPI, ROW>::STAGES;
    constexpr bool kTma = EPI == RBK_EPI_STORE_F16 || EPI == RBK_EPI_BIAS_GELU || EPI == RBK_EPI_GELU_BWD;
    constexpr int kWarpStage = PairEpi<EPI, ROW>::WARP_STAGE;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = su32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw);
    const uint32_t sA0 = base;
    const uint32_t epi_stage = base + STAGES * STAGE_BYTES;
    const uint32_t part_s = epi_stage + kEpiWarps * kWarpStage;      // ROW: float [kRowWarps][BM]
    const uint32_t bars = part_s + PairEpi<EPI, ROW>::PART_BYTES;
    uint8_t* gbars = gbase + (bars - base);
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (STAGES + s); };
    auto tfull_bar = [&](int b) { return bars + 8u * (2 * STAGES + b); };
    auto tempty_bar = [&](int b) { return bars + 8u * (2 * STAGES + 2 + b); };
    auto consumed_bar = [&](int s) { return bars + 8u * (2 * STAGES + 4 + s); };   // ROW only
    const uint32_t parts_rdy = bars + 8u * (3 * STAGES + 4);                   // ROW: partials written
    const uint32_t parts_free = parts_rdy + 8u;                                 // ROW: partials read
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbars + 8 * (3 * STAGES + 6));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gbars + 8 * (3 * STAGES + 6) + 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;
    constexpr bool kRowWarp = EPI == RBK_EPI_ACC_F32 && ROW;
    constexpr int nbuf = 2;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
            if (kRowWarp) mbar_init(consumed_bar(s), 1);
        }
        if (kRowWarp) {
            mbar_init(parts_rdy, kRowWarps);
            mbar_init(parts_free, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), 2 * kEpiWarps);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0 && lane == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, 512);
    fence_before();
    __syncthreads();
    cluster_sync();                                  // the peer's barriers are initialised
    fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_dependency_sync();

    if (warp == 0) {
        // ------------------------------ TMA producer (both CTAs) -------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int u = pair; u < p.units && !*abort_flag; u += num_pairs) {
                int mb, nb, kb0, kb1;
                decode_unit(p, u, mb, nb, kb0, kb1);
                const int m0 = mb * 2 * BM + (int)rank * BM, n0 = nb * BN + (int)rank * HALF_N;
                bool ok = true;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag)) { ok = false; break; }
                    if (leader) mbar_expect_tx(full_bar(stage), 2 * STAGE_BYTES);
                    const uint32_t fb = mapa_shared(full_bar(stage), 0);
                    const uint32_t sa = sA0 + stage * STAGE_BYTES;
                    const uint32_t sb = sa + A_BYTES;
                    const int k0 = kb * BK;
                    if (!p.a_mn) {
                        tma_load_2d_pair(sa, &tmA, fb, k0, m0);
                    } else {
                        tma_load_2d_pair(sa, &tmA, fb, m0, k0);
                        tma_load_2d_pair(sa + 8192, &tmA, fb, m0 + 64, k0);
                    }
                    if (!p.b_mn) {
                        tma_load_2d_pair(sb, &tmB, fb, k0, n0);
                    } else {
                        tma_load_2d_pair(sb, &tmB, fb, n0, k0);
                        tma_load_2d_pair(sb + 8192, &tmB, fb, n0 + 64, k0);
                    }
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
                if (!ok) break;
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer (even CTA) ----------------
        if (leader && lane == 0) {
            const uint32_t idesc = idesc_f16_m256(BN, p.a_mn, p.b_mn);
            const uint32_t a_lbo = p.a_mn ? 8192u : 16u, b_lbo = p.b_mn ? 8192u : 16u;
            const uint32_t a_kstep = p.a_mn ? 2048u : 32u, b_kstep = p.b_mn ? 2048u : 32u;
            int stage = 0, buf = 0;
            uint32_t phase = 0, bphase = 0;
            for (int u = pair; u < p.units && !*abort_flag; u += num_pairs) {
                int mb, nb, kb0, kb1;
                decode_unit(p, u, mb, nb, kb0, kb1);
                const bool rows_tile = kRowWarp && p.dbias_rows != nullptr && nb == 0;
                if (!mbar_wait(tempty_bar(buf), bphase ^ 1, abort_flag)) break;
                fence_after();
                const uint32_t dacc = tmem + buf * BN;
                bool ok = true;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(full_bar(stage), phase, abort_flag)) { ok = false; break; }
                    fence_after();
                    const uint32_t sa = sA0 + stage * STAGE_BYTES;
                    const uint32_t sb = sa + A_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; ++k) {
                        const uint32_t acc = (kb > kb0 || k > 0) ? 1u : 0u;
                        mma_f16_pair(dacc, sdesc(sa + k * a_kstep, a_lbo, 1024), sdesc(sb + k * b_kstep, b_lbo, 1024),
                                     idesc, acc);
                    }
                    // the stage is consumed: free it (row-sum tiles: the stage's row warp in each CTA
                    // reads it first)
                    const uint32_t rel = rows_tile ? consumed_bar(stage) : empty_bar(stage);
                    mma_commit_pair(rel);
                    mma_commit_pair(mapa_shared(rel, 1));
                    if (++stage == STAGES) { stage = 0; phase ^= 1; }
                }
                if (!ok) break;
                mma_commit_pair(tfull_bar(buf));
                mma_commit_pair(mapa_shared(tfull_bar(buf), 1));
                if (++buf == nbuf) { buf = 0; bphase ^= 1; }
            }
        }
    } else if (kRowWarp && warp >= 2 + kEpiWarps) {
        // ------------------------------ row sums of A (both CTAs) ------------
        // Row warp rw owns the operand stages s % kRowWarps == rw.  On the tiles of n block 0 every use of
        // them passes through here after the MMAs have read it: the CTA's 128 rows of A over the
        // stage's 64 k are added into FP32 sums, then the stage is freed for the producer.
        const int rw = warp - 2 - kEpiWarps;
        float* part = reinterpret_cast<float*>(gbase + (part_s - base));
        uint32_t j = 0;                                  // k blocks of this pair so far (all tiles)
        static_assert(STAGES <= 2 * kRowWarps, "a row warp owns at most two stages");
        uint32_t uses0 = 0, uses1 = 0;                   // row-tile uses of the two owned stages
        uint32_t rphase = 0;                             // row-sum tiles so far (hand-off parity)
        bool ok = true;
        for (int u = pair; ok && u < p.units; u += num_pairs) {
            int mb, nb, kb0, kb1;
            decode_unit(p, u, mb, nb, kb0, kb1);
            const bool rows = p.dbias_rows != nullptr && nb == 0;
            if (!rows) {                                 // its stages are freed by the MMA thread
                j += (uint32_t)(kb1 - kb0);
                continue;
            }
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (int kb = kb0; kb < kb1; ++kb, ++j) {
                const int stage = (int)(j % STAGES);
                if (stage % kRowWarps != rw) continue;
                const bool second = stage >= kRowWarps;
                const uint32_t n = second ? uses1++ : uses0++;
                // the MMAs have read the stage (their commit follows the TMA's completion of it)
                ok = __all_sync(0xffffffffu, mbar_wait(consumed_bar(stage), n & 1, abort_flag));
                if (!ok) break;
                {
                    fence_proxy_async();                    // the TMA (async proxy) wrote the stage
                    const uint32_t sa = sA0 + stage * STAGE_BYTES;
                    if (p.a_mn) {
                        // two boxes of 64 rows (k) x 128 B (64 m); 16-byte chunk c of row k sits at
                        // c ^ (k & 7).  Lane l: the 8 m of chunk l % 8 of box (l / 8) % 2, rows
                        // k = 32 (l / 16) .. + 31
                        const uint32_t box = sa + (uint32_t)((lane >> 3) & 1) * 8192u;
                        const uint32_t c = (uint32_t)(lane & 7), k0 = (uint32_t)(lane >> 4) * 32u;
#pragma unroll 8
                        for (uint32_t k = k0; k < k0 + 32u; ++k) {
                            const uint4 v = lds128(box + k * 128u + ((c ^ (k & 7u)) << 4));
                            add_f16x2(acc[0], acc[1], v.x);
                            add_f16x2(acc[2], acc[3], v.y);
                            add_f16x2(acc[4], acc[5], v.z);
                            add_f16x2(acc[6], acc[7], v.w);
                        }
                    } else {
                        // 128 rows (m) x 128 B (64 k); chunk c of row m at c ^ (m & 7).  Lane l: rows
                        // l + 32 i, i < 4 (sums in acc[i])
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint32_t m = (uint32_t)(lane + 32 * i);
                            float s0 = 0.f, s1 = 0.f;
#pragma unroll
                            for (uint32_t c = 0; c < 8; ++c) {
                                const uint4 v = lds128(sa + m * 128u + ((c ^ (m & 7u)) << 4));
                                add_f16x2(s0, s1, v.x);
                                add_f16x2(s0, s1, v.y);
                                add_f16x2(s0, s1, v.z);
                                add_f16x2(s0, s1, v.w);
                            }
                            acc[i] += s0 + s1;
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty_bar(stage));   // the producer may refill the stage
            }
            if (!ok) break;
            // this warp's partial sums of the tile's 128 rows -> part[rw][*]
            if (p.a_mn) {
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], 16);   // both k halves
            }
            ok = __all_sync(0xffffffffu, mbar_wait(parts_free, (rphase & 1) ^ 1, abort_flag));
            if (!ok) break;
            if (p.a_mn) {
                if (lane < 16) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) part[rw * BM + 8 * lane + e] = acc[e];
                }
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) part[rw * BM + lane + 32 * i] = acc[i];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(parts_rdy);
            if (rw == 0) {
                // the partials in warp order, then this rank's 128 rows of dbias
                ok = __all_sync(0xffffffffu, mbar_wait(parts_rdy, rphase & 1, abort_flag));
                if (ok) {
                    const int split = u % p.splits;
                    const int mode = acc_mode(p, split);
                    const int mbase = mb * 2 * BM + (int)rank * BM;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int r = lane + 32 * i, m = mbase + r;
                        float v = part[r];
#pragma unroll
                        for (int w = 1; w < kRowWarps; ++w) v += part[w * BM + r];
                        if (m < p.M) {
                            const float bv = p.alpha * v;
                            if (mode == kAccPlane) p.part_rows[(size_t)(split - 1) * p.M + m] = bv;
                            else if (mode == kAccOwner) p.dbias_rows[m] += bv;
                            else atomicAdd(p.dbias_rows + m, bv);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(parts_free);
                }
            }
            ++rphase;
        }
    } else {
        // ------------------------------ epilogue (both CTAs) -----------------
        const int q = warp & 3;
        const int half_id = (warp - 2) / 4;
        constexpr int kChunks = BN / 32;
        const int c0 = half_id * (kChunks / 2), c1 = half_id ? kChunks : kChunks / 2;
        uint8_t* my_stage = gbase + (epi_stage - base) + (warp - 2) * kWarpStage;
        const uint32_t my_stage_s = epi_stage + (warp - 2) * kWarpStage;
        int sc = 0;
        int buf = 0;
        uint32_t bphase = 0;
        for (int u = pair; u < p.units; u += num_pairs) {
            int mb, nb, kb0, kb1;
            decode_unit(p, u, mb, nb, kb0, kb1);
            const int m0 = mb * 2 * BM + (int)rank * BM + q * 32;
            const int split = u % p.splits;
            const int mode = acc_mode(p, split);
            constexpr bool kAux = EPI == RBK_EPI_STORE_F16 || EPI == RBK_EPI_BIAS_GELU || EPI == RBK_EPI_GELU_BWD;
            constexpr bool kOwn = EPI == RBK_EPI_ACC_F32;        // C values the owner adds to, one chunk ahead
            const bool own = kOwn && mode == kAccOwner;
            const int lda = p.ld_aux ? p.ld_aux : p.ldc;
            uint4 pf[4];
            float4 cpf[kOwn ? 8 : 1];
            if (kAux && p.aux) prefetch_h(pf, p.aux, lda, m0, nb * BN + c0 * 32, p, lane);
            if constexpr (kOwn) {
                if (own) load_c_row(cpf, p, m0, nb * BN + c0 * 32, lane);
            }
            if (!mbar_wait(tfull_bar(buf), bphase, abort_flag)) break;
            fence_after();
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + buf * BN;
#pragma unroll 1
            for (int c = c0; c < c1; ++c) {
                uint32_t r[32];
                tmem_ld32(tbase + c * 32, r);
                uint4 cur[4] = {pf[0], pf[1], pf[2], pf[3]};
                if (kAux && p.aux && c + 1 < c1) prefetch_h(pf, p.aux, lda, m0, nb * BN + (c + 1) * 32, p, lane);
                tmem_wait_ld();
                if constexpr (kTma) {
                    epilogue_chunk_tma<EPI>(p, m0, nb * BN + c * 32, r, my_stage, my_stage_s, lane, cur, &tmC, &tmX, sc);
                } else {
                    float4 cv[kOwn ? 8 : 1];
                    if constexpr (kOwn) {
#pragma unroll
                        for (int k = 0; k < 8; ++k) cv[k] = cpf[k];
                        if (own && c + 1 < c1) load_c_row(cpf, p, m0, nb * BN + (c + 1) * 32, lane);
                    }
                    epilogue_chunk_f32_tma<EPI>(p, m0, nb * BN + c * 32, r, my_stage, my_stage_s, lane, &tmC, &tmP,
                                                split, mode, cv);
                }
            }
            // the accumulator reads are complete (tcgen05.wait::ld); the tile's global stores need not
            // drain before the MMAs may reuse the buffer, so the arrival is relaxed
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster_relaxed(mapa_shared(tempty_bar(buf), 0));
            if (++buf == nbuf) { buf = 0; bphase ^= 1; }
        }
        if (lane == 0) bulk_wait0();                       // tensor stores / reduce-adds complete before exit
    }

    fence_before();
    __syncthreads();
    cluster_sync();                                  // no remote arrival or commit is still in flight
    fence_after();
    if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, RBK_ERR_TIMEOUT);
    if (warp == 1) tmem_free_pair(tmem, 512);
}

// ------------------------------------------------------------------- host ----
template <int BN, int EPI>
int launch(rbk_ctx* ctx, const rbk_gemm_desc* d, Params& p, cudaStream_t st) {
    using C = Cfg<BN>;
    CUtensorMap ta, tb;
    if (!d->a_major) RBK_TRY(make_tmap(&ta, d->A, d->K, d->M, d->lda, 64, 128));
    else RBK_TRY(make_tmap(&ta, d->A, d->M, d->K, d->lda, 64, 64));
    if (!d->b_major) RBK_TRY(make_tmap(&tb, d->B, d->K, d->N, d->ldb, 64, BN));
    else RBK_TRY(make_tmap(&tb, d->B, d->N, d->K, d->ldb, 64, 64));
    static int configured_device = -1;   // attribute is per device; one device per process
    if (configured_device != ctx->device) {
        RBK_CUDA(cudaFuncSetAttribute(gemm_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        configured_device = ctx->device;
    }
    int grid = p.units < ctx->num_sms ? p.units : ctx->num_sms;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cfg.numAttrs = set_pdl(attr, 0);
    cfg.attrs = attr;
    RBK_CUDA(cudaLaunchKernelEx(&cfg, gemm_kernel<BN, EPI>, ta, tb, p));
    RBK_LAUNCHED("gemm_kernel");
    return RBK_OK;
}

// Launched as 2-CTA clusters; grid = 2 x min(units, pairs that fit at once).
template <int EPI, bool ROW = false>
int launch_pair(rbk_ctx* ctx, const rbk_gemm_desc* d, Params& p, cudaStream_t st) {
    constexpr int SMEM = PairEpi<EPI, ROW>::SMEM;
    static_assert(SMEM <= 232448, "shared memory budget");
    CUtensorMap ta, tb, tc_, tx, tp;
    // FP16 outputs: 32 x 32 store boxes over the logical [M, N] (ldc / ld_aux pitches); FP32
    // outputs: 16 x 32 boxes (64-byte rows), the split planes of deterministic mode a 3-D map
    constexpr bool kTma = EPI == RBK_EPI_STORE_F16 || EPI == RBK_EPI_BIAS_GELU || EPI == RBK_EPI_GELU_BWD;
    memset(&tc_, 0, sizeof(tc_));
    memset(&tx, 0, sizeof(tx));
    memset(&tp, 0, sizeof(tp));
    if (kTma) {
        if (d->C)
            RBK_TRY(make_tmap(&tc_, d->C, d->N, d->M, d->ldc, 32, 32, CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                              CU_TENSOR_MAP_SWIZZLE_64B));
        if (EPI == RBK_EPI_BIAS_GELU)
            RBK_TRY(make_tmap(&tx, d->aux_out, d->N, d->M, d->ld_aux ? d->ld_aux : d->ldc, 32, 32,
                              CU_TENSOR_MAP_DATA_TYPE_FLOAT16, CU_TENSOR_MAP_SWIZZLE_64B));
    } else {
        RBK_TRY(make_tmap(&tc_, d->C, d->N, d->M, d->ldc, 16, 32, CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                          CU_TENSOR_MAP_SWIZZLE_64B));
        if (p.part) RBK_TRY(make_tmap_3d(&tp, p.part, d->N, d->M, p.splits - 1, p.ldp, 16, 32));
    }
    if (!d->a_major) RBK_TRY(make_tmap(&ta, d->A, d->K, d->M, d->lda, 64, 128));
    else RBK_TRY(make_tmap(&ta, d->A, d->M, d->K, d->lda, 64, 64));
    if (!d->b_major) RBK_TRY(make_tmap(&tb, d->B, d->K, d->N, d->ldb, 64, 128));
    else RBK_TRY(make_tmap(&tb, d->B, d->N, d->K, d->ldb, 64, 64));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(PairEpi<EPI, ROW>::THREADS);
    cfg.dynamicSmemBytes = SMEM;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    static int configured_device = -1, max_pairs = 0;
    if (configured_device != ctx->device) {
        RBK_CUDA(cudaFuncSetAttribute(gemm_pair_kernel<EPI, ROW>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        cfg.gridDim = dim3(ctx->num_sms & ~1);
        int n = 0;
        RBK_CUDA(cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<EPI, ROW>, &cfg));
        max_pairs = n > 0 ? n : ctx->num_sms / 2;
        configured_device = ctx->device;
    }
    const int pairs = p.units < max_pairs ? p.units : max_pairs;
    cfg.gridDim = dim3(2 * pairs);
    cfg.numAttrs = set_pdl(attr, 1);
    RBK_CUDA(cudaLaunchKernelEx(&cfg, gemm_pair_kernel<EPI, ROW>, ta, tb, tc_, tx, tp, p));
    RBK_LAUNCHED("gemm_pair_kernel");
    return RBK_OK;
}

// CTA pairs unless RBK_GEMM_SINGLE=1 (the 1-CTA kernel for every N = 256 problem).
static bool pair_tiles() {
    static const int v = [] {
        const char* e = getenv("RBK_GEMM_SINGLE");
        return (e && e[0] == '1') ? 0 : 1;
    }();
    return v != 0;
}

}  // namespace gemm
}  // namespace rbk

using namespace rbk;
using namespace rbk::gemm;

extern "C" {

int rbk_gemm(rbk_ctx* ctx, const rbk_gemm_desc* d, void* stream) {
    RBK_REQUIRE(ctx && d && d->A && d->B && (d->C || (d->epilogue == RBK_EPI_BIAS_GELU && d->aux_out)),
                "rbk_gemm: null pointer");
    RBK_REQUIRE(d->M > 0 && d->N > 0 && d->K > 0, "rbk_gemm: empty problem (M=%d N=%d K=%d)", d->M, d->N, d->K);
    RBK_REQUIRE(d->epilogue >= RBK_EPI_STORE_F16 && d->epilogue <= RBK_EPI_STORE_F32, "rbk_gemm: bad epilogue");
    RBK_REQUIRE(d->lda % 8 == 0 && d->ldb % 8 == 0 && d->ldc % 8 == 0 && (d->ld_aux % 8 == 0),
                "rbk_gemm: leading dimensions must be multiples of 8 elements");
    RBK_REQUIRE(aligned16(d->A) && aligned16(d->B) && aligned16(d->C) && (!d->aux || aligned16(d->aux)) &&
                    (!d->aux_out || aligned16(d->aux_out)) && (!d->bias || aligned16(d->bias)),
                "rbk_gemm: pointers must be 16-byte aligned");
    RBK_REQUIRE(d->lda >= (d->a_major ? d->M : d->K) && d->ldb >= (d->b_major ? d->N : d->K),
                "rbk_gemm: leading dimension smaller than the contiguous extent");
    RBK_REQUIRE(d->epilogue != RBK_EPI_BIAS_GELU || (d->bias && d->aux_out), "rbk_gemm: BIAS_GELU needs bias and aux_out");
    RBK_REQUIRE(d->epilogue != RBK_EPI_GELU_BWD || d->aux, "rbk_gemm: GELU_BWD needs aux (pre-activation)");
    RBK_REQUIRE(!d->dbias_rows || d->epilogue == RBK_EPI_ACC_F32, "rbk_gemm: dbias_rows needs ACC_F32");
    int epi = d->epilogue;
    // Tile width: N=256 tiles amortise each A tile over the most MMA columns; the
    // wgrad with a fused bias gradient uses N=192 so that two accumulators plus
    // the ones-MMA accumulator fit the 512 TMEM columns; narrow problems use 128.
    int BN;
    if (epi == RBK_EPI_ACC_F32)
        BN = d->N <= 128 ? 128 : d->N < 256 ? 192 : (d->dbias_rows && !pair_tiles()) ? 192 : 256;
    else
        BN = d->N >= 512 ? 256 : 128;
    // N = 256 problems run on CTA pairs (256 x 256 pair tiles)
    const bool pair = BN == 256 && pair_tiles();
    const int slots = pair ? ctx->num_sms / 2 : ctx->num_sms;
    Params p;
    p.M = d->M; p.N = d->N; p.K = d->K;
    p.m_blocks = (d->M + (pair ? 2 * BM : BM) - 1) / (pair ? 2 * BM : BM);
    p.n_blocks = (d->N + BN - 1) / BN;
    p.k_blocks = (d->K + BK - 1) / BK;
    int splits = 1;
    if (epi == RBK_EPI_ACC_F32) {
        // Split K (FP32 accumulation makes the splits add up) so the persistent
        // grid's waves are nearly full: take the fewest splits whose wave
        // efficiency units / (ceil(units / SMs) * SMs) is >= 90%, else the best.
        const int tiles = p.m_blocks * p.n_blocks;
        const int max_split = p.k_blocks / 8 > 0 ? p.k_blocks / 8 : 1;
        // A destination known to hold zeros (and no row sums) is written by one unit per tile
        // with the plain FP32 store epilogue: about 1.1-1.35x the rate of reduce-added split-K
        // partials on the 1.3B weight gradients, so it keeps one split unless the grid's last
        // wave would be less than 80% full.
        const long w1 = (tiles + slots - 1) / slots;
        const bool store_one = ctx->gemm_c_zero && !d->dbias_rows && BN != 192 &&
                               (double)tiles / (double)(w1 * slots) >= 0.8;
        if (d->split_k > 0) {
            splits = d->split_k;
        } else if (store_one) {
            splits = 1;
        } else {
            double best = -1.0;
            for (int s = 1; s <= max_split && s <= 64; ++s) {
                const int kbps = (p.k_blocks + s - 1) / s;
                const int real = (p.k_blocks + kbps - 1) / kbps;
                const long units = (long)tiles * real;
                const long waves = (units + slots - 1) / slots;
                const double eff = (double)units / (double)(waves * slots);
                if (eff > best + 1e-9) { best = eff; splits = s; }
                if (eff >= 0.9) break;
            }
        }
        if (splits > max_split) splits = max_split;
        if (splits < 1) splits = 1;
    }
    p.kb_per_split = (p.k_blocks + splits - 1) / splits;
    p.splits = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;
    // C + acc = acc: the store epilogue (no read of C, fewer registers than the accumulating one)
    if (epi == RBK_EPI_ACC_F32 && ctx->gemm_c_zero && p.splits == 1 && !d->dbias_rows && BN != 192)
        epi = RBK_EPI_STORE_F32;
    p.units = p.m_blocks * p.n_blocks * p.splits;
    p.a_mn = d->a_major ? 1 : 0;
    p.b_mn = d->b_major ? 1 : 0;
    p.C = d->C; p.ldc = d->ldc;
    p.bias = (const half*)d->bias;
    p.aux = (const half*)d->aux;
    p.ld_aux = d->ld_aux;
    p.aux_out = (half*)d->aux_out;
    p.dbias_rows = d->dbias_rows;
    p.alpha = d->alpha;
    p.err = ctx->tickets + kGemmError;
    p.part = nullptr;
    p.part_rows = nullptr;
    p.ldp = (d->N + 3) & ~3;
    p.c_zero = epi == RBK_EPI_ACC_F32 && ctx->gemm_c_zero;
    const bool det = epi == RBK_EPI_ACC_F32 && p.splits > 1 && ctx->deterministic;
    if (det) {
        // one FP32 plane per split after the first (+ its row sums), added to C in split order
        // after the GEMM; split 0 adds its tile to C itself
        const size_t plane = (size_t)d->M * p.ldp;
        void* ws;
        RBK_TRY(ctx_scratch(ctx, sizeof(float) * ((p.splits - 1) * plane + (size_t)(p.splits - 1) * d->M), &ws));
        p.part = static_cast<float*>(ws);
        p.part_rows = p.part + (p.splits - 1) * plane;
    }
    cudaStream_t st = as_stream(stream);
    const int role = ctx->gemm_role >= 0 ? ctx->gemm_role
                     : (epi == RBK_EPI_ACC_F32 || epi == RBK_EPI_STORE_F32) ? 2 : d->b_major ? 1 : 0;
    ProfScope prof(ctx, st, kCatGemm, 2.0 * d->M * (double)d->N * d->K, role);
    auto run = [&]() -> int {
        if (pair) {
            switch (epi) {
                case RBK_EPI_STORE_F16: return launch_pair<RBK_EPI_STORE_F16>(ctx, d, p, st);
                case RBK_EPI_BIAS_GELU: return launch_pair<RBK_EPI_BIAS_GELU>(ctx, d, p, st);
                case RBK_EPI_GELU_BWD: return launch_pair<RBK_EPI_GELU_BWD>(ctx, d, p, st);
                case RBK_EPI_ACC_F32:
                    return d->dbias_rows ? launch_pair<RBK_EPI_ACC_F32, true>(ctx, d, p, st)
                                         : launch_pair<RBK_EPI_ACC_F32, false>(ctx, d, p, st);
                default: return launch_pair<RBK_EPI_STORE_F32>(ctx, d, p, st);
            }
        }
        if (BN == 256) {
            switch (epi) {
                case RBK_EPI_STORE_F16: return launch<256, RBK_EPI_STORE_F16>(ctx, d, p, st);
                case RBK_EPI_BIAS_GELU: return launch<256, RBK_EPI_BIAS_GELU>(ctx, d, p, st);
                case RBK_EPI_GELU_BWD: return launch<256, RBK_EPI_GELU_BWD>(ctx, d, p, st);
                case RBK_EPI_ACC_F32: return launch<256, RBK_EPI_ACC_F32>(ctx, d, p, st);
                default: return launch<256, RBK_EPI_STORE_F32>(ctx, d, p, st);
            }
        }
        if (BN == 192) return launch<192, RBK_EPI_ACC_F32>(ctx, d, p, st);
        switch (epi) {
            case RBK_EPI_STORE_F16: return launch<128, RBK_EPI_STORE_F16>(ctx, d, p, st);
            case RBK_EPI_BIAS_GELU: return launch<128, RBK_EPI_BIAS_GELU>(ctx, d, p, st);
            case RBK_EPI_GELU_BWD: return launch<128, RBK_EPI_GELU_BWD>(ctx, d, p, st);
            case RBK_EPI_ACC_F32: return launch<128, RBK_EPI_ACC_F32>(ctx, d, p, st);
            default: return launch<128, RBK_EPI_STORE_F32>(ctx, d, p, st);
        }
    };
    RBK_TRY(run());
    if (det) {
        const size_t work = (size_t)d->M * ((d->N + 3) / 4);
        const size_t want = (work + 255) / 256;
        const int blocks = (int)(want < (size_t)ctx->num_sms * 8 ? want : (size_t)ctx->num_sms * 8);
        RBK_CUDA(launch_pdl(splitk_reduce_kernel, dim3(blocks), dim3(256), 0, st, (float*)d->C, d->ldc,
                            (const float*)p.part, d->M, d->N, p.ldp, p.splits - 1, d->dbias_rows,
                            (const float*)p.part_rows));
        RBK_LAUNCHED("splitk_reduce_kernel");
    }
    return RBK_OK;
}

int rbk_linear_fwd(rbk_ctx* ctx, void* Y, const void* X, const void* W, const void* bias, const void* residual,
                   int N, int in, int out, void* stream) {
    rbk_gemm_desc d = {};
    d.M = N; d.N = out; d.K = in;
    d.A = X; d.lda = in; d.a_major = 0;
    d.B = W; d.ldb = in; d.b_major = 0;
    d.C = Y; d.ldc = out;
    d.epilogue = RBK_EPI_STORE_F16;
    d.bias = bias;
    d.aux = residual;
    d.alpha = 1.0f;
    return rbk_gemm(ctx, &d, stream);
}

int rbk_gemm_dgrad(rbk_ctx* ctx, void* dX, const void* dY, const void* W, int N, int in, int out,
                   const void* gelu_pre, void* stream) {
    rbk_gemm_desc d = {};
    d.M = N; d.N = in; d.K = out;
    d.A = dY; d.lda = out; d.a_major = 0;
    d.B = W; d.ldb = in; d.b_major = 1;      // B(n=in, k=out) = W[out, in]
    d.C = dX; d.ldc = in;
    d.epilogue = gelu_pre ? RBK_EPI_GELU_BWD : RBK_EPI_STORE_F16;
    d.aux = gelu_pre;
    d.alpha = 1.0f;
    return rbk_gemm(ctx, &d, stream);
}

int rbk_gemm_wgrad(rbk_ctx* ctx, float* dW, float* dbias, const void* dY, const void* X, int N, int in, int out,
                   void* stream) {
    rbk_gemm_desc d = {};
    d.M = out; d.N = in; d.K = N;
    d.A = dY; d.lda = out; d.a_major = 1;    // A(m=out, k=token) = dY[token, out]
    d.B = X; d.ldb = in; d.b_major = 1;      // B(n=in, k=token) = X[token, in]
    d.C = dW; d.ldc = in;
    d.epilogue = RBK_EPI_ACC_F32;
    d.dbias_rows = dbias;
    d.alpha = 1.0f;
    return rbk_gemm(ctx, &d, stream);
}

}  // extern "C"
