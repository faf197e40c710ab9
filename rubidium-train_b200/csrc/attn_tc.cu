// attn_tc.cu — causal flash attention forward on the 5th-generation tensor
// cores (d_head 64 or 128): the tcgen05 replacement of the mma.sync forward in
// attn.cu for sequence lengths that are multiples of 128.
//
// One CTA = one (batch, head, 128-query block); at d_head 64 two CTAs share an
// SM.  Keys are consumed 64 at a time.  Q and K tiles are d_head/64 128B-swizzle
// atoms wide (one TMA box each), V is d_head/64 MN-major column blocks, O is
// d_head TMEM columns.  Roles (192 threads):
//   warp 0     TMA: Q once (128 x 64 box), K through a 3-stage ring and V
//              through a 2-stage ring (64 x 64 boxes), all from the fused
//              q|k|v rows of the QKV projection
//   warp 1     MMA: S_j = Q K_j^T into one of two TMEM buffers (128 x 64 FP32),
//              so S_{j+1} is computed while the softmax works on S_j; then
//              O += P_j V_j into TMEM (128 x 64 FP32) with P_j from shared memory
//   warps 2-5  softmax (P double-buffered: no wait on the PV just issued),
//              one query row per thread (TMEM lane = row: the row max
//              and sum need no cross-thread reduction); P = exp2(S*scale*log2e
//              - m) goes to shared memory as FP16 in the 128B-swizzled K-major
//              layout the PV MMA reads.  O is rescaled only when a row max grows
//              by more than 2^8 (P stays <= 256, within FP16 range).
// Causal masking applies to the two key blocks that overlap the query block;
// blocks above the diagonal are never loaded.  Output O (FP16) and LSE
// (natural log), as the mma.sync path.  Every wait is bounded; no multicast.
#include "tc.cuh"

namespace rbk {
namespace attn_tc {

using namespace tc;

constexpr int BQ = 128, BKV = 64;
constexpr int kThreads = 192;
template <int HD>
struct FwdCfg {
    static constexpr int NA = HD / 64;                  // 64-column atoms across d_head
    static constexpr int KS = HD == 64 ? 4 : 3, VS = HD == 64 ? 3 : 3;   // K / V ring depths
    static constexpr int Q_BYTES = BQ * HD * 2;         // NA atoms of 16 KB
    static constexpr int KV_BYTES = BKV * HD * 2;       // NA atoms of 8 KB
    static constexpr int P_BYTES = BQ * BKV * 2;        // 16 KB: one 64-key K-major atom
    static constexpr int OFF_Q = 0, OFF_K = OFF_Q + Q_BYTES, OFF_V = OFF_K + KS * KV_BYTES,
                         OFF_P = OFF_V + VS * KV_BYTES;
    static constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;   // P double-buffered
    static constexpr int SMEM = 1024 + OFF_BAR + 256;
    static constexpr int CTAS_PER_SM = HD == 64 ? 2 : 1;
};
constexpr uint32_t TMEM_COLS = 256;       // S0 [0, 64), S1 [64, 128), O [128, 128 + d_head)
constexpr uint32_t O_COL = 128;

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int HD>
__global__ void __launch_bounds__(kThreads, FwdCfg<HD>::CTAS_PER_SM)
    flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmkv, half* O,
                        float* LSE, int S, int H, float scale_log2, int* err) {
    using Cf = FwdCfg<HD>;
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
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;

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
            const uint32_t o_tm = tmem + O_COL;
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
#pragma unroll
                for (int k = 0; k < BKV / 16; ++k)
                    mma_f16(o_tm, sdesc(sP(j & 1) + k * 32, 16, 1024),
                            sdesc(sV(vs) + k * 2048, BKV * 128, 1024),   // N blocks of 64 columns, 8 KB apart
                            idesc_o, (j > 0 || k > 0) ? 1u : 0u);
                mma_commit(o_done(j & 1));
                mma_commit(v_empty(vs));
                if (j + 2 < nkv && !issue_s(j + 2)) break;   // S buffer j&1 was released by p_full[j&1]
            }
        }
    } else {
        // ------------------------------------------------------ softmax ----
        const int q4 = warp & 3;
        const int row = q4 * 32 + lane;                   // query row inside the block
        const int qpos = qb * BQ + row;                   // query position in the sequence
        const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
        float m = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
            if (!mbar_wait(s_full(j & 1), (j >> 1) & 1, abort_flag)) { ok = false; break; }
            fence_after();
            const bool mask = (j + 1) * BKV > qb * BQ;   // block overlaps the diagonal region
            uint32_t r[64];
            tmem_ld32(tmem + lane_off + (uint32_t)(j & 1) * BKV, r);
            tmem_ld32(tmem + lane_off + (uint32_t)(j & 1) * BKV + 32, r + 32);
            tmem_wait_ld();
            // eight independent max / sum accumulators: no 64-long dependency chains
            float x[64];
            float mxp[8];
#pragma unroll
            for (int a = 0; a < 8; ++a) mxp[a] = -INFINITY;
            const int lim = mask ? qpos - j * BKV : 1 << 30;   // keys e > lim are masked
#pragma unroll
            for (int e = 0; e < 64; ++e) {
                const float v = e > lim ? -INFINITY : __uint_as_float(r[e]) * scale_log2;
                x[e] = v;
                mxp[e & 7] = fmaxf(mxp[e & 7], v);
            }
            const float mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                                   fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
            float corr = 1.0f;
            bool rescale = false;
            if (mx > m + 8.0f) {                          // lazy rescale (first block: m = -inf)
                if (j > 0) { corr = ex2(m - mx); rescale = true; }
                m = mx;
                l *= corr;
            }
            float p[64];
            float rsp[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int e = 0; e < 64; ++e) {
                p[e] = ex2(x[e] - m);
                rsp[e & 7] += p[e];
            }
            l += ((rsp[0] + rsp[1]) + (rsp[2] + rsp[3])) + ((rsp[4] + rsp[5]) + (rsp[6] + rsp[7]));
            // P buffer j&1 was last read by PV_{j-2}
            if (j > 1) {
                if (!mbar_wait(o_done(j & 1), ((j >> 1) & 1) ^ 1, abort_flag)) { ok = false; break; }
                fence_after();
            }
            if (__any_sync(0xffffffffu, rescale)) {
                // O must hold every earlier PV before it is rescaled: wait for PV_{j-1}
                if (!mbar_wait(o_done((j - 1) & 1), ((j - 1) >> 1) & 1, abort_flag)) { ok = false; break; }
                fence_after();
#pragma unroll
                for (int c = 0; c < HD / 32; ++c) {
                    uint32_t t[32];
                    tmem_ld32(tmem + lane_off + O_COL + c * 32, t);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) t[e] = __float_as_uint(__uint_as_float(t[e]) * corr);
                    tmem_st32(tmem + lane_off + O_COL + c * 32, t);
                }
                tmem_wait_st();
            }
#pragma unroll
            for (int c = 0; c < 8; ++c) {                 // 16-byte chunk = 8 keys, 128B swizzle
                const uint32_t addr = sP(j & 1) + (uint32_t)row * 128u + (uint32_t)((c ^ (row & 7)) << 4);
                const uint4 u = f_to_h8(p + 8 * c);
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(u.x), "r"(u.y), "r"(u.z),
                             "r"(u.w)
                             : "memory");
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full(j & 1));
        }
        // epilogue: O / l (FP16) and LSE
        if (ok && mbar_wait(o_done((nkv - 1) & 1), ((nkv - 1) >> 1) & 1, abort_flag)) {
            fence_after();
            const float inv = 1.0f / l;
            half* orow = O + ((size_t)row0 + qpos) * D + h * HD;
#pragma unroll
            for (int c = 0; c < HD / 32; ++c) {
                uint32_t t[32];
                tmem_ld32(tmem + lane_off + O_COL + c * 32, t);
                tmem_wait_ld();
                float o[32];
#pragma unroll
                for (int e = 0; e < 32; ++e) o[e] = __uint_as_float(t[e]) * inv;
#pragma unroll
                for (int g = 0; g < 4; ++g) reinterpret_cast<uint4*>(orow + c * 32)[g] = f_to_h8(o + 8 * g);
            }
            LSE[(size_t)bh * S + qpos] = (m + __log2f(l)) * 0.6931471805599453f;
        }
    }
    fence_before();
    __syncthreads();
    fence_after();
    if (threadIdx.x == 0 && *abort_flag) atomicExch(err, RBK_ERR_TIMEOUT);
    if (warp == 1) tmem_free(tmem, TMEM_COLS);
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
    flash_fwd_tc_kernel<HD><<<grid, kThreads, FwdCfg<HD>::SMEM, st>>>(
        tmq, tmkv, (half*)o, lse, S, H, scale * 1.4426950408889634f, ctx->tickets + kGemmError);
    RBK_LAUNCHED("flash_fwd_tc_kernel");
    return RBK_OK;
}

int attn_fwd_tc(rbk_ctx* ctx, void* o, float* lse, const void* qkv, int B, int S, int H, int dh, float scale,
                cudaStream_t st) {
    return dh == 64 ? attn_fwd_tc_hd<64>(ctx, o, lse, qkv, B, S, H, scale, st)
                    : attn_fwd_tc_hd<128>(ctx, o, lse, qkv, B, S, H, scale, st);
}

}  // namespace rbk
