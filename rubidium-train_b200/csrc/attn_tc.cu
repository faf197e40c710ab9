// attn_tc.cu — causal flash attention forward on the 5th-generation tensor
// cores (d_head 64 or 128): the tcgen05 replacement of the mma.sync forward in
// attn.cu for sequence lengths that are multiples of 128.
//
// One CTA = one (batch, head, 128-query block); at d_head 64 two CTAs share an
// SM.  Keys are consumed 64 at a time.  Q and K tiles are d_head/64 128B-swizzle
// atoms wide (one TMA box each), V is d_head/64 MN-major column blocks.  Two
// softmax warpgroups take alternate key blocks, each with its own running row
// max / sum and its own O accumulator in TMEM; the two partial results are
// merged at the end (O = O0 2^(m0-m) + O1 2^(m1-m), l likewise).  That doubles
// the warps working through the exp / max / sum chains, which bound the
// kernel, at the same TMEM budget.  Roles (320 threads):
//   warp 0     TMA: Q once (128 x 64 box), K through a KS-stage ring and V
//              through a VS-stage ring (64 x 64 boxes), all from the fused
//              q|k|v rows of the QKV projection
//   warp 1     MMA: S_j = Q K_j^T into TMEM buffer j & 1 (128 x 64 FP32), then
//              O_{j&1} += P_j V_j with P_j from shared memory
//   warps 2-5  softmax, even key blocks; warps 6-9 odd key blocks.  One query
//              row per thread (TMEM lane = row: the row max and sum need no
//              cross-thread reduction); P = exp2(S*scale*log2e - m) is one FFMA
//              and one ex2 per score and goes to shared memory as FP16 in the
//              128B-swizzled K-major layout the PV MMA reads.  A group rescales
//              its O only when its row max grows by more than 2^8 (P <= 256,
//              within FP16 range).
// TMEM: S0 [0, 64), S1 [64, 128), O0 [128, 128 + d_head), O1 after O0.
// Causal masking applies to the two key blocks that overlap the query block;
// blocks above the diagonal are never loaded.  Output O (FP16) and LSE
// (natural log), as the mma.sync path.  Every wait is bounded; no multicast.
#include "tc.cuh"

namespace rbk {
namespace attn_tc {

using namespace tc;

constexpr int BQ = 128, BKV = 64;
template <int HD>
struct FwdCfg {
    static constexpr int NA = HD / 64;                  // 64-column atoms across d_head
    static constexpr int KS = HD == 64 ? 4 : 3, VS = HD == 64 ? 3 : 3;   // K / V ring depths
    static constexpr int Q_BYTES = BQ * HD * 2;         // NA atoms of 16 KB
    static constexpr int KV_BYTES = BKV * HD * 2;       // NA atoms of 8 KB
    static constexpr int P_BYTES = BQ * BKV * 2;        // 16 KB: one 64-key K-major atom
    static constexpr int OFF_Q = 0, OFF_K = OFF_Q + Q_BYTES, OFF_V = OFF_K + KS * KV_BYTES,
                         OFF_P = OFF_V + VS * KV_BYTES;
    static constexpr int OFF_ML = OFF_P + 2 * P_BYTES;    // P double-buffered; then (m, l) of both groups
    static constexpr int OFF_BAR = OFF_ML + 2 * BQ * 8;
    static constexpr int SMEM = 1024 + OFF_BAR + 256;
    static constexpr int CTAS_PER_SM = HD == 64 ? 2 : 1;
    // softmax groups: two at d_head 128 (one CTA per SM); one at d_head 64, where two CTAs share
    // an SM and a second group's registers would not fit
    static constexpr int NG = HD == 64 ? 1 : 2;
    static constexpr int THREADS = 64 + 128 * NG;
    static constexpr uint32_t TMEM_COLS = HD == 64 ? 256 : 512;   // S0, S1, O0 (, O1)
};
constexpr uint32_t O_COL = 128;

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
template <int HD>
__global__ void __launch_bounds__(FwdCfg<HD>::THREADS, FwdCfg<HD>::CTAS_PER_SM)
    flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmkv, half* O,
                        float* LSE, int S, int H, float scale_log2, int* err) {
    using Cf = FwdCfg<HD>;
    constexpr int NG = Cf::NG;
    constexpr int NA = Cf::NA, KS = Cf::KS, VS = Cf::VS, Q_BYTES = Cf::Q_BYTES, KV_BYTES = Cf::KV_BYTES,
                  P_BYTES = Cf::P_BYTES, OFF_Q = Cf::OFF_Q, OFF_K = Cf::OFF_K, OFF_V = Cf::OFF_V, OFF_P = Cf::OFF_P,
                  OFF_BAR = Cf::OFF_BAR;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = su32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw);
    const uint32_t sQ = base + OFF_Q;
    auto sP = [&](int s) { return base + OFF_P + (uint32_t)s * P_BYTES; };
    auto sK = [&](int s) { return base + OFF_K + (uint32_t)s * KV_BYTES; };
    auto sV = [&](int s) { return base + OFF_V + (uint32_t)s * KV_BYTES; };
    // barriers: q_full | k_full[KS] | k_empty[KS] | v_full[VS] | v_empty[VS] | s_full[2] | p_full[2] |
    // o_done[2] (one barrier per buffer, so a wait never targets a phase two completions old)
    const uint32_t bars = base + OFF_BAR;
    const uint32_t q_full = bars;
    auto k_full = [&](int s) { return bars + 8 + 8 * s; };
    auto k_empty = [&](int s) { return bars + 8 + 8 * KS + 8 * s; };
    auto v_full = [&](int s) { return bars + 8 + 16 * KS + 8 * s; };
    auto v_empty = [&](int s) { return bars + 8 + 16 * KS + 8 * VS + 8 * s; };
    const uint32_t bars2 = bars + 8 + 16 * KS + 16 * VS;
    auto s_full = [&](int s) { return bars2 + 8 * s; };
    auto p_full = [&](int s) { return bars2 + 16 + 8 * s; };
    auto o_done = [&](int s) { return bars2 + 32 + 8 * s; };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (bars2 - base) + 48);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + (bars2 - base) + 56);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nqb = S / BQ;
    const int qb = nqb - 1 - (int)blockIdx.x;     // longest rows first
    const int bh = blockIdx.y, b = bh / H, h = bh % H;
    const int D = H * HD;
    const int row0 = b * S;
    const int nkv = (qb + 1) * (BQ / BKV);       // key blocks up to the diagonal

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < KS; ++s) { mbar_init(k_full(s), 1); mbar_init(k_empty(s), 1); }
        for (int s = 0; s < VS; ++s) { mbar_init(v_full(s), 1); mbar_init(v_empty(s), 1); }
        mbar_init(s_full(0), 1); mbar_init(s_full(1), 1);
        for (int s = 0; s < 2; ++s) { mbar_init(p_full(s), 4); mbar_init(o_done(s), 1); }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0 && lane == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmq) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmkv) : "memory");
    }
    if (warp == 1) tmem_alloc(tmem_slot, Cf::TMEM_COLS);
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_dependency_sync();

    if (warp == 0) {
        // ---------------------------------------------------------- TMA ----
        // lane 0 streams Q then K, lane 16 streams V: the two rings refill independently
        if (lane == 0) {
            mbar_expect_tx(q_full, Q_BYTES);
#pragma unroll
            for (int a = 0; a < NA; ++a) tma_load_2d(sQ + a * (BQ * 128), &tmq, q_full, h * HD + 64 * a, row0 + qb * BQ);
            for (int j = 0; j < nkv; ++j) {
                const int ks = j % KS;
                if (!mbar_wait(k_empty(ks), ((j / KS) & 1) ^ 1, abort_flag)) break;
                mbar_expect_tx(k_full(ks), KV_BYTES);
#pragma unroll
                for (int a = 0; a < NA; ++a)
                    tma_load_2d(sK(ks) + a * (BKV * 128), &tmkv, k_full(ks), D + h * HD + 64 * a, row0 + j * BKV);
            }
        } else if (lane == 16) {
            for (int j = 0; j < nkv; ++j) {
                const int vs = j % VS;
                if (!mbar_wait(v_empty(vs), ((j / VS) & 1) ^ 1, abort_flag)) break;
                mbar_expect_tx(v_full(vs), KV_BYTES);
#pragma unroll
                for (int a = 0; a < NA; ++a)
                    tma_load_2d(sV(vs) + a * (BKV * 128), &tmkv, v_full(vs), 2 * D + h * HD + 64 * a, row0 + j * BKV);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA ----
        if (lane == 0) {
            const uint32_t idesc_s = idesc_f16(BKV, 0, 0);   // Q (K-major) x K (K-major), N = 64
            const uint32_t idesc_o = idesc_f16(HD, 0, 1);    // P (K-major) x V (MN-major), N = d_head
            auto issue_s = [&](int j) -> bool {
                const int ks = j % KS;
                if (!mbar_wait(k_full(ks), (j / KS) & 1, abort_flag)) return false;
                fence_after();
                const uint32_t s_tm = tmem + (uint32_t)(j & 1) * BKV;
#pragma unroll
                for (int k = 0; k < HD / 16; ++k)   // K = d_head: atom k / 4, 32 B per step inside it
                    mma_f16(s_tm, sdesc(sQ + (k >> 2) * (BQ * 128) + (k & 3) * 32, 16, 1024),
                            sdesc(sK(ks) + (k >> 2) * (BKV * 128) + (k & 3) * 32, 16, 1024), idesc_s, k > 0);
                mma_commit(s_full(j & 1));
                mma_commit(k_empty(ks));
                return true;
            };
            bool ok = mbar_wait(q_full, 0, abort_flag) && issue_s(0) && (nkv < 2 || issue_s(1));
            for (int j = 0; ok && j < nkv; ++j) {
                const int vs = j % VS;
                if (!mbar_wait(p_full(j & 1), (j >> 1) & 1, abort_flag) ||
                    !mbar_wait(v_full(vs), (j / VS) & 1, abort_flag))
                    break;
                fence_after();
                const uint32_t o_tm = tmem + O_COL + (NG == 2 ? (uint32_t)(j & 1) * HD : 0u);   // the group's O
#pragma unroll
                for (int k = 0; k < BKV / 16; ++k)
                    mma_f16(o_tm, sdesc(sP(j & 1) + k * 32, 16, 1024),
                            sdesc(sV(vs) + k * 2048, BKV * 128, 1024),   // N blocks of 64 columns, 8 KB apart
                            idesc_o, (j >= NG || k > 0) ? 1u : 0u);
                mma_commit(o_done(j & 1));
                mma_commit(v_empty(vs));
                if (j + 2 < nkv && !issue_s(j + 2)) break;   // S buffer j&1 was released by p_full[j&1]
            }
        }
    } else {
        // ------------------------------------------------------ softmax ----
        const int wg = NG == 2 ? (warp - 2) >> 2 : 0;    // two groups: even / odd key blocks
        const int q4 = warp & 3;
        const int row = q4 * 32 + lane;                   // query row inside the block
        const int qpos = qb * BQ + row;                   // query position in the sequence
        const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
        const uint32_t o_col = O_COL + (uint32_t)wg * HD;
        float m = -INFINITY, l = 0.0f;                    // running max (log2 units) and sum of this group
        bool ok = true;
        int jl = 0;                                       // blocks of this group done
        for (int j = wg; j < nkv; j += NG, ++jl) {
            const int sb = j & 1;                         // S / P buffer of block j
            if (!mbar_wait(s_full(sb), (j >> 1) & 1, abort_flag)) { ok = false; break; }
            fence_after();
            const bool mask = (j + 1) * BKV > qb * BQ;   // block overlaps the diagonal region
            uint32_t r[64];
            tmem_ld32(tmem + lane_off + (uint32_t)sb * BKV, r);
            tmem_ld32(tmem + lane_off + (uint32_t)sb * BKV + 32, r + 32);
            tmem_wait_ld();
            // four independent max accumulators, two scores per 3-input max
            float mxp[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) mxp[a] = -INFINITY;
            if (mask) {
                const int lim = qpos - j * BKV;           // keys e > lim are masked
#pragma unroll
                for (int e = 0; e < 64; ++e)
                    if (e > lim) r[e] = __float_as_uint(-INFINITY);
            }
#pragma unroll
            for (int e = 0; e < 64; e += 2)
                mxp[(e >> 1) & 3] = fmax3(mxp[(e >> 1) & 3], __uint_as_float(r[e]), __uint_as_float(r[e + 1]));
            const float mx = scale_log2 * fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3]));
            float corr = 1.0f;
            bool rescale = false;
            if (mx > m + 8.0f) {                          // lazy rescale (first block: m = -inf)
                if (jl > 0) { corr = ex2(m - mx); rescale = true; }
                m = mx;
                l *= corr;
            }
            // P buffer sb (and, with two groups, O_wg) was last read by PV_{j-2}
            if (j > 1) {
                if (!mbar_wait(o_done(sb), ((j >> 1) & 1) ^ 1, abort_flag)) { ok = false; break; }
                fence_after();
            }
            if (__any_sync(0xffffffffu, rescale)) {
                if constexpr (NG == 1) {                  // the single O must hold PV_{j-1} before its rescale
                    if (!mbar_wait(o_done((j - 1) & 1), ((j - 1) >> 1) & 1, abort_flag)) { ok = false; break; }
                    fence_after();
                }
#pragma unroll 1
                for (int c = 0; c < HD / 16; ++c) {
                    uint32_t t[16];
                    tmem_ld16(tmem + lane_off + o_col + c * 16, t);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; ++e) t[e] = __float_as_uint(__uint_as_float(t[e]) * corr);
                    tmem_st16(tmem + lane_off + o_col + c * 16, t);
                }
                tmem_wait_st();
            }
            // p = 2^(s * scale * log2 e - m); a row with no visible key yet keeps m = -inf and p = 0.
            // Each 16-byte chunk of 8 keys goes to shared memory as soon as it is packed.
            const float nm = m == -INFINITY ? 0.0f : -m;
            const uint64_t c2 = pair_of(scale_log2), nm2 = pair_of(nm);
            uint64_t rs2[2] = {0, 0};                     // two packed (even, odd) sum accumulators
#pragma unroll
            for (int c = 0; c < 8; ++c) {                 // 16-byte chunk = 8 keys, 128B swizzle
                uint32_t pk[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int e = 8 * c + 2 * q;
                    float x0, x1;
                    ffma2(x0, x1, __uint_as_float(r[e]), __uint_as_float(r[e + 1]), c2, nm2);
                    const float p0 = ex2(x0), p1 = ex2(x1);
                    fadd2(rs2[q & 1], p0, p1);
                    __half2 hp = __floats2half2_rn(p0, p1);
                    pk[q] = *reinterpret_cast<uint32_t*>(&hp);
                }
                const uint32_t addr = sP(sb) + (uint32_t)row * 128u + (uint32_t)((c ^ (row & 7)) << 4);
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pk[0]), "r"(pk[1]), "r"(pk[2]),
                             "r"(pk[3])
                             : "memory");
            }
            l += (__uint_as_float((uint32_t)rs2[0]) + __uint_as_float((uint32_t)(rs2[0] >> 32))) +
                 (__uint_as_float((uint32_t)rs2[1]) + __uint_as_float((uint32_t)(rs2[1] >> 32)));
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full(sb));
        }
        // epilogue.  One group: O / l.  Two groups: after each has seen its last PV, swap (m, l)
        // and each writes half of the columns of
        // O = (O0 2^(m0-M) + O1 2^(m1-M)) / (l0 2^(m0-M) + l1 2^(m1-M)).
        const int jlast = nkv - NG + wg;                  // last block of this group (nkv is even)
        ok = ok && mbar_wait(o_done(jlast & 1), (jlast >> 1) & 1, abort_flag);
        float f0 = 0.0f, f1 = 0.0f, M = m, L = l;
        if constexpr (NG == 2) {
            float* ml = reinterpret_cast<float*>(gbase + Cf::OFF_ML);
            ml[(wg * BQ + row) * 2] = m;
            ml[(wg * BQ + row) * 2 + 1] = l;
            fence_before();
            named_sync(1, 256);
            fence_after();
            ok = ok && !*abort_flag;
            const float m0 = ml[row * 2], l0 = ml[row * 2 + 1];
            const float m1 = ml[(BQ + row) * 2], l1 = ml[(BQ + row) * 2 + 1];
            M = fmaxf(m0, m1);
            const float a0 = m0 == -INFINITY ? 0.0f : ex2(m0 - M), a1 = m1 == -INFINITY ? 0.0f : ex2(m1 - M);
            L = l0 * a0 + l1 * a1;
            f0 = a0 / L;
            f1 = a1 / L;
        } else {
            f0 = 1.0f / l;
        }
        if (ok) {
            half* orow = O + ((size_t)row0 + qpos) * D + h * HD;
#pragma unroll 1
            for (int c = wg * (HD / 16 / NG); c < (wg + 1) * (HD / 16 / NG); ++c) {   // 16 columns at a time
                uint32_t t0[16], t1[16];
                tmem_ld16(tmem + lane_off + O_COL + c * 16, t0);
                if constexpr (NG == 2) tmem_ld16(tmem + lane_off + O_COL + HD + c * 16, t1);
                tmem_wait_ld();
                float o[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    o[e] = __uint_as_float(t0[e]) * f0;
                    if constexpr (NG == 2) o[e] = fmaf(__uint_as_float(t1[e]), f1, o[e]);
                }
#pragma unroll
                for (int g = 0; g < 2; ++g) reinterpret_cast<uint4*>(orow + c * 16)[g] = f_to_h8(o + 8 * g);
            }
            if (wg == 0) LSE[(size_t)bh * S + qpos] = (M + __log2f(L)) * 0.6931471805599453f;
        }
    }
    fence_before();
    __syncthreads();
    fence_after();
    if (threadIdx.x == 0 && *abort_flag) atomicExch(err, RBK_ERR_TIMEOUT);
    if (warp == 1) tmem_free(tmem, Cf::TMEM_COLS);
}

}  // namespace attn_tc

// Used by rbk_attn_fwd (attn.cu) when d_head is 64 or 128 and S % 128 == 0.
template <int HD>
static int attn_fwd_tc_hd(rbk_ctx* ctx, void* o, float* lse, const void* qkv, int B, int S, int H, float scale,
                          cudaStream_t st) {
    using namespace attn_tc;
    const int D = H * HD;
    CUtensorMap tmq, tmkv;
    RBK_TRY(tc::make_tmap(&tmq, qkv, 3 * (uint64_t)D, (uint64_t)B * S, 3 * (uint64_t)D, 64, BQ));
    RBK_TRY(tc::make_tmap(&tmkv, qkv, 3 * (uint64_t)D, (uint64_t)B * S, 3 * (uint64_t)D, 64, BKV));
    static int set_dev = -1;
    if (set_dev != ctx->device) {
        RBK_CUDA(cudaFuncSetAttribute(flash_fwd_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      FwdCfg<HD>::SMEM));
        set_dev = ctx->device;
    }
    dim3 grid(S / BQ, B * H);
    RBK_CUDA(launch_pdl(flash_fwd_tc_kernel<HD>, grid, dim3(FwdCfg<HD>::THREADS), FwdCfg<HD>::SMEM, st, tmq, tmkv,
                        (half*)o, lse, S, H, scale * 1.4426950408889634f, ctx->tickets + kGemmError));
    RBK_LAUNCHED("flash_fwd_tc_kernel");
    return RBK_OK;
}

int attn_fwd_tc(rbk_ctx* ctx, void* o, float* lse, const void* qkv, int B, int S, int H, int dh, float scale,
                cudaStream_t st) {
    return dh == 64 ? attn_fwd_tc_hd<64>(ctx, o, lse, qkv, B, S, H, scale, st)
                    : attn_fwd_tc_hd<128>(ctx, o, lse, qkv, B, S, H, scale, st);
}

}  // namespace rbk
