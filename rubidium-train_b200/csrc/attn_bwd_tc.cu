// attn_bwd_tc.cu — causal flash attention backward on the 5th-generation
// tensor cores (d_head 64 or 128, sequence length a multiple of 128): the
// tcgen05 replacement of the mma.sync main kernel in attn.cu.  The pre pass
// (Dot = rowsum(dO * O), -LSE * log2 e, zeroed FP32 dQ accumulator) and the
// post pass (dQ -> FP16, q- and v-bias column sums) are shared with the
// mma.sync path.
//
// d_head 64.  Work item = one (batch, head, 128-key block): it walks the
// 128-query sub-tiles from the diagonal to the end of the sequence.  Per
// sub-tile i (TMEM lane = key, column = query):
//   S^T_i  = K Q_i^T          dP^T_i = V dO_i^T       (M = N = 128, K = 64)
//   P^T_i  = exp2(S^T * scale * log2 e - LSE * log2 e)     (0 above the diagonal)
//   dS^T_i = P^T_i * (dP^T_i - Dot)
//   dV    += P^T_i dO_i       dK    += dS^T_i Q_i     (K = 128 queries)
//   dQ_i   = dS_i K           (M = 128 queries, K = 128 keys) -> TMA reduce-add
// into the FP32 accumulator.  P^T goes back to TMEM as FP16 and is the A
// operand of the dV product straight from there; dS^T goes to shared memory as
// FP16 in the 128B-swizzled layout: K-major for the dK product and, read the
// other way, MN-major for the dQ product, so one copy serves both.  Once dQ_i
// is in TMEM, the dS^T_i tile is the FP32 staging buffer of its reduce-add.
// 128-query sub-tiles make every product an N = 128 or K = 128 MMA and halve
// the hand-offs between the issuing threads and the P / dS warps per FLOP;
// TMEM holds exactly one of each: S^T 0, dP^T 128, P^T 256 (FP16 pairs),
// dK 320, dV 384, dQ 448.
//
// The kernel is persistent: one CTA per SM takes work items round-robin from
// a longest-first order; K and V are double-buffered so the next item's tiles
// load while the current one finishes, and the dK / dV epilogue of one item
// overlaps the start of the next: the accumulators are read out of TMEM as
// FP16 into the item's own K / V tiles (no longer needed once its last MMA is
// done) and leave by TMA store.
//
// Roles (736 threads):
//   warp 0       TMA: K and V per item, then Q_i, dO_i and the per-query rows
//                (-LSE log2 e, Dot) through a 2-stage ring
//   warp 1       MMA issue, producer side: S^T_i and dP^T_i
//   warp 2       MMA issue, consumer side: dV, dK and dQ.  Two issuing
//                threads in different warps: a single issuer that also waits
//                on barriers leaves the tensor pipe idle for each wait.
//   warps 3-18   P / dS: warp w owns TMEM lanes 32 (w % 4) .. +31 and query
//                columns 32 ((w - 3) / 4) .. +31 of each sub-tile, in two
//                halves of 16
//   warps 19-22  dQ drain (TMEM -> swizzled FP32 staging -> reduce-add), then
//                the dK / dV epilogue of each item (TMEM -> K / V tiles -> TMA
//                store)
// Every wait is bounded; no cluster multicast.
//
// d_head 128 (attn_tc_bwd128 below) keeps 64-query sub-tiles: dK and dV alone
// take 256 TMEM columns there.
//
// Bias gradients: the key bias has an exactly zero gradient (it shifts every
// score of a query row by the same amount, and sum_j dS_ij = Dot_i - Dot_i = 0),
// and the value bias gradient is sum_j dV_j = sum_i dO_i (rows of P sum to 1);
// the post pass adds the latter from dO, so these kernels write no bias terms.
#include "tc.cuh"

namespace rbk {
namespace attn_tc_bwd {

using namespace tc;

constexpr int BK = 128, BQ = 128, HD = 64;
constexpr int QS = 3;                       // Q / dO ring depth
constexpr int NE = 16;                      // P / dS warps
constexpr int WE = 3;                       // first P / dS warp
constexpr int WD = WE + NE;                 // first drain warp
constexpr int kThreads = (WD + 4) * 32;
constexpr int KT_BYTES = BK * HD * 2;       // 16 KB  K or V block
constexpr int QT_BYTES = BQ * HD * 2;       // 16 KB  Q or dO sub-tile
constexpr int PT_BYTES = BK * BQ * 2;       // 32 KB  dS^T sub-tile: two 64-query atoms of 16 KB
constexpr int PA_BYTES = BK * 128;          // one atom of dS^T
constexpr int ROW_BYTES = 2 * BQ * 4;       // -LSE log2e | Dot of one sub-tile
constexpr int STG_BYTES = BQ * 32 * 4;      // 16 KB  FP32 dQ staging: 128 queries x 32 columns (one box)
constexpr int OFF_K = 0, OFF_V = OFF_K + 2 * KT_BYTES, OFF_Q = OFF_V + 2 * KT_BYTES, OFF_DO = OFF_Q + QS * QT_BYTES,
              OFF_DS = OFF_DO + QS * QT_BYTES, OFF_STG = OFF_DS + PT_BYTES, OFF_ROW = OFF_STG + STG_BYTES,
              OFF_BAR = OFF_ROW + QS * ROW_BYTES;
constexpr int NBARS = 2 * QS + 4 + 2 + 2 + 2 + 2 + 2;
constexpr int SMEM = 1024 + OFF_BAR + NBARS * 8 + 16;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t S_COL = 0, DP_COL = 128, P_COL = 256, DK_COL = 320, DV_COL = 384, DQ_COL = 448;
static_assert(SMEM <= 232448, "shared memory budget");

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ float4 ld_shared_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

// FP32 [128 rows][64 cols] staging as two 128B-swizzled boxes of 32 columns.
__device__ __forceinline__ uint32_t stage_addr(uint32_t s, int row, int chunk /* 16 B = 4 floats, 0..15 */) {
    return s + (uint32_t)(chunk >> 3) * 16384u + (uint32_t)row * 128u + (uint32_t)(((chunk & 7) ^ (row & 7)) << 4);
}

// Deterministic dQ (dq_sem != nullptr): the contributions to a query block are added in
// ascending key-block order.  dq_sem counts, per (batch * head, 64-query block), the
// contributions already added; an item waits until the count shows every lower key block done.
// Items are dispatched key-block-major (lower key blocks first) to CTAs that are all resident,
// so the item waited on is already running or done; every wait is bounded.
__device__ __forceinline__ int ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __noinline__ bool wait_count(const int* p, int want, volatile int* abort_flag) {
    if (ld_acquire(p) >= want) return true;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire(p) < want) {
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
            *abort_flag = 1;
            return false;
        }
        __nanosleep(128);
    }
    return true;
}
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Work item u (longest first: all diagonal-0 key blocks, then 1, ...).
struct Item {
    int kb, bh, h, n, krow0;
};
__device__ __forceinline__ Item item_of(int u, int BH, int H, int S) {
    Item it;
    it.kb = u / BH;
    it.bh = u % BH;
    it.h = it.bh % H;
    it.n = (S - it.kb * BK) / 64;         // 64-query sub-tiles from the diagonal to S (d_head 128)
    it.krow0 = (it.bh / H) * S + it.kb * BK;
    return it;
}

struct Masked {
    static constexpr bool value = true;
};
struct Plain {
    static constexpr bool value = false;
};

__global__ void __launch_bounds__(kThreads, 1)
    flash_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmkv,
                        const __grid_constant__ CUtensorMap tmdo, const __grid_constant__ CUtensorMap tmdq,
                        const __grid_constant__ CUtensorMap tmout, const float* __restrict__ NL2,
                        const float* __restrict__ Dot, int S, int H, int num_items, float scale, float scale_log2,
                        int* err, int* __restrict__ dq_sem, const __grid_constant__ CUtensorMap tmdq64,
                        const __grid_constant__ CUtensorMap tmout64) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = su32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw);
    auto sK = [&](int s) { return base + OFF_K + (uint32_t)s * KT_BYTES; };
    auto sV = [&](int s) { return base + OFF_V + (uint32_t)s * KT_BYTES; };
    auto sQ = [&](int s) { return base + OFF_Q + (uint32_t)s * QT_BYTES; };
    auto sdO = [&](int s) { return base + OFF_DO + (uint32_t)s * QT_BYTES; };
    auto sRow = [&](int s) { return base + OFF_ROW + (uint32_t)s * ROW_BYTES; };
    const uint32_t sdS = base + OFF_DS, sStg = base + OFF_STG;
    // barriers
    const uint32_t bars = base + OFF_BAR;
    auto q_full = [&](int s) { return bars + 8 * s; };
    auto q_empty = [&](int s) { return bars + 8 * QS + 8 * s; };
    const uint32_t b2 = bars + 16 * QS;
    auto kv_full = [&](int s) { return b2 + 8 * s; };       // K, V of an item in buffer s
    auto kv_empty = [&](int s) { return b2 + 16 + 8 * s; }; // K / V buffer s free: producer done, dK / dV stored
    const uint32_t s_full = b2 + 32, s_free = b2 + 40;      // S^T, dP^T in TMEM / loaded by the P / dS warps
    const uint32_t p_full = b2 + 48, p_free = b2 + 56;      // P^T in TMEM and dS^T in smem / P^T read by dV
    const uint32_t ds_free = b2 + 64;                       // dS^T read by dK and dQ: reusable
    const uint32_t dq_full = b2 + 72, dq_free = b2 + 80, acc_done = b2 + 88, acc_free = b2 + 96;
    const uint32_t ds_full = b2 + 104;                      // dS^T in shared memory
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_BAR + NBARS * 8);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + OFF_BAR + NBARS * 8 + 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkb = (S + BK - 1) / BK;
    const int BH = num_items / nkb;
    const bool half_tail = S % BK != 0;     // the last key / query block holds 64 rows
    const int D = H * HD;
    // sub-tiles of item u: 128-query blocks from the diagonal to the end
    auto subtiles = [&](int u) { return nkb - u / BH; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < QS; ++s) {
            mbar_init(q_full(s), 1);
            mbar_init(q_empty(s), NE + 2);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(kv_full(s), 1);
            mbar_init(kv_empty(s), 2);
        }
        mbar_init(ds_free, 1);
        mbar_init(ds_full, NE);
        mbar_init(s_full, 1);
        mbar_init(s_free, NE);
        mbar_init(p_full, NE);
        mbar_init(p_free, 1);
        mbar_init(dq_full, 1);
        mbar_init(dq_free, 4);
        mbar_init(acc_done, 1);
        mbar_init(acc_free, 4);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0 && lane == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmq) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmkv) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmdo) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmdq) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmout) : "memory");
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_dependency_sync();

    if (warp == 0) {
        // ---------------------------------------------------------- TMA ----
        if (lane == 0) {
            int g = 0;                                       // sub-tile counter of this CTA
            bool ok = true;
            for (int t = 0, u = blockIdx.x; ok && u < num_items; ++t, u += gridDim.x) {
                const Item it = item_of(u, BH, H, S);
                const int n = subtiles(u);
                const int kvb = t & 1;
                if (!mbar_wait(kv_empty(kvb), ((t >> 1) & 1) ^ 1, abort_flag)) break;
                mbar_expect_tx(kv_full(kvb), 2 * KT_BYTES);
                tma_load_2d(sK(kvb), &tmkv, kv_full(kvb), D + it.h * HD, it.krow0);
                tma_load_2d(sV(kvb), &tmkv, kv_full(kvb), 2 * D + it.h * HD, it.krow0);
                const float* nl2 = NL2 + (size_t)it.bh * S + it.kb * BK;
                const float* dot = Dot + (size_t)it.bh * S + it.kb * BK;
                for (int i = 0; i < n; ++i, ++g) {
                    const int s = g % QS;
                    if (!mbar_wait(q_empty(s), ((g / QS) & 1) ^ 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = q_full(s);
                    mbar_expect_tx(fb, 2 * QT_BYTES + ROW_BYTES);
                    tma_load_2d(sQ(s), &tmq, fb, it.h * HD, it.krow0 + i * BQ);
                    tma_load_2d(sdO(s), &tmdo, fb, it.h * HD, it.krow0 + i * BQ);
                    bulk_load(sRow(s), nl2 + i * BQ, BQ * 4, fb);
                    bulk_load(sRow(s) + BQ * 4, dot + i * BQ, BQ * 4, fb);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------- MMA: S^T, dP^T producer ----
        if (lane == 0) {
            const uint32_t id_s = idesc_f16(BQ, 0, 0);    // K (K-major) x Q^T (K-major): N = 128 queries
            int g = 0;
            bool ok = true;
            for (int t = 0, u = blockIdx.x; ok && u < num_items; ++t, u += gridDim.x) {
                const int n = subtiles(u);
                const int kvb = t & 1;
                if (!mbar_wait(kv_full(kvb), (t >> 1) & 1, abort_flag)) break;
                for (int i = 0; i < n; ++i, ++g) {
                    const int s = g % QS;
                    ok = mbar_wait(q_full(s), (g / QS) & 1, abort_flag) &&
                         (g == 0 || mbar_wait(s_free, (g - 1) & 1, abort_flag));
                    if (!ok) break;
                    fence_after();
#pragma unroll
                    for (int k = 0; k < HD / 16; ++k)
                        mma_f16(tmem + S_COL, sdesc(sK(kvb) + k * 32, 16, 1024), sdesc(sQ(s) + k * 32, 16, 1024), id_s,
                                k > 0);
#pragma unroll
                    for (int k = 0; k < HD / 16; ++k)
                        mma_f16(tmem + DP_COL, sdesc(sV(kvb) + k * 32, 16, 1024), sdesc(sdO(s) + k * 32, 16, 1024),
                                id_s, k > 0);
                    mma_commit(s_full);
                    mma_commit(q_empty(s));
                }
                if (ok) mma_commit(kv_empty(kvb));
            }
        }
    } else if (warp == 2) {
        // ------------------------------------------- MMA: dV, dK, dQ consumer ----
        if (lane == 0) {
            const uint32_t id_kv = idesc_f16(HD, 0, 1);   // P^T (TMEM) / dS^T (K-major) x dO / Q (MN-major): N = 64
            const uint32_t id_q = idesc_f16(HD, 1, 1);    // dS (MN-major) x K (MN-major): N = 64
            int g = 0;
            bool ok = true;
            for (int t = 0, u = blockIdx.x; ok && u < num_items; ++t, u += gridDim.x) {
                const int n = subtiles(u);
                const int kvb = t & 1;
                // K is an operand of dQ; the accumulators must have been read out for the previous item
                ok = mbar_wait(kv_full(kvb), (t >> 1) & 1, abort_flag) &&
                     (t == 0 || mbar_wait(acc_free, (t - 1) & 1, abort_flag));
                if (!ok) break;
                for (int i = 0; i < n; ++i, ++g) {
                    const int s = g % QS;
                    const uint32_t ds = sdS;
                    // dK and dQ need only dS^T (shared memory): they run while P^T is still being stored
                    if (!mbar_wait(ds_full, g & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    fence_after();
#pragma unroll
                    for (int k = 0; k < BQ / 16; ++k)
                        mma_f16(tmem + DK_COL, sdesc(ds + (k >> 2) * PA_BYTES + (k & 3) * 32, 16, 1024),
                                sdesc(sQ(s) + k * 2048, 8192, 1024), id_kv, (i > 0 || k > 0) ? 1u : 0u);
                    if (g > 0 && !mbar_wait(dq_free, (g - 1) & 1, abort_flag)) {   // dQ_{g-1} read out of TMEM
                        ok = false;
                        break;
                    }
                    fence_after();
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        mma_f16(tmem + DQ_COL, sdesc(ds + k * 2048, PA_BYTES, 1024), sdesc(sK(kvb) + k * 2048, 8192, 1024),
                                id_q, k > 0);
                    mma_commit(dq_full);
                    mma_commit(ds_free);
                    if (!mbar_wait(p_full, g & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    fence_after();
#pragma unroll
                    for (int k = 0; k < BQ / 16; ++k)
                        mma_f16_ts(tmem + DV_COL, tmem + P_COL + (uint32_t)(k * 8), sdesc(sdO(s) + k * 2048, 8192, 1024),
                                   id_kv, (i > 0 || k > 0) ? 1u : 0u);
                    mma_commit(p_free);
                    mma_commit(q_empty(s));
                }
                if (ok) mma_commit(acc_done);
            }
        }
    } else if (warp < WD) {
        // ------------------------------------------------------ P / dS ----
        const int lg = warp & 3, cg = (warp - WE) >> 2;
        const int r = lg * 32 + lane;                         // key row inside the block
        const uint32_t lane_off = (uint32_t)(lg * 32) << 16;
        const int c0 = cg * 32;                               // first query column of this warp
        const uint64_t c2 = pair_of(scale_log2);
        int g = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < num_items; u += gridDim.x) {
            const int n = subtiles(u);
            const int kbu = u / BH;                            // the item's key block
            for (int i = 0; i < n; ++i, ++g) {
                const int s = g % QS;
                ok = mbar_wait(s_full, g & 1, abort_flag) && mbar_wait(q_full(s), (g / QS) & 1, abort_flag);
                if (!__all_sync(0xffffffffu, ok)) {
                    ok = false;
                    break;
                }
                fence_after();
                const uint32_t rowp = sRow(s);
                uint32_t pk[16], dk[16];
                // query columns at or beyond qmax lie past the sequence end (a half last block): P = 0
                const int qmax = S - (kbu * BK + i * BQ) - c0;
                // columns c0 + 16 h .. +15; masked: the diagonal sub-tile, where columns e < lim lie above it
                auto compute = [&](auto masked, auto tail, int h, const uint32_t* sr, const uint32_t* dr) {
                    const int lim = r - c0 - 16 * h;
                    const int qm = qmax - 16 * h;
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const int cc = c0 + 16 * h + 4 * q4;
                        const float4 nl = ld_shared_f4(rowp + (uint32_t)cc * 4);
                        const float4 dt = ld_shared_f4(rowp + BQ * 4 + (uint32_t)cc * 4);
                        const float nlv[4] = {nl.x, nl.y, nl.z, nl.w}, dtv[4] = {dt.x, dt.y, dt.z, dt.w};
                        float pv[4], dv[4];
#pragma unroll
                        for (int e4 = 0; e4 < 4; e4 += 2) {       // packed FP32 pairs
                            const int e = 4 * q4 + e4;
                            float x0, x1;
                            ffma2v(x0, x1, __uint_as_float(sr[e]), __uint_as_float(sr[e + 1]), c2, nlv[e4],
                                   nlv[e4 + 1]);
                            float p0 = ex2(x0), p1 = ex2(x1);
                            if (decltype(masked)::value) {
                                p0 = e < lim ? 0.0f : p0;
                                p1 = e + 1 < lim ? 0.0f : p1;
                            }
                            if (decltype(tail)::value) {
                                p0 = e >= qm ? 0.0f : p0;
                                p1 = e + 1 >= qm ? 0.0f : p1;
                            }
                            pv[e4] = p0;
                            pv[e4 + 1] = p1;
                            float d0, d1;
                            fsub2(d0, d1, __uint_as_float(dr[e]), __uint_as_float(dr[e + 1]), dtv[e4], dtv[e4 + 1]);
                            fmul2(dv[e4], dv[e4 + 1], p0, p1, d0, d1);
                        }
                        pk[8 * h + 2 * q4] = pack_h2(pv[0], pv[1]);
                        pk[8 * h + 2 * q4 + 1] = pack_h2(pv[2], pv[3]);
                        dk[8 * h + 2 * q4] = pack_h2(dv[0], dv[1]);
                        dk[8 * h + 2 * q4 + 1] = pack_h2(dv[2], dv[3]);
                    }
                };
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t sr[16], dr[16];
                    tmem_ld16(tmem + lane_off + S_COL + c0 + 16 * h, sr);
                    tmem_ld16(tmem + lane_off + DP_COL + c0 + 16 * h, dr);
                    tmem_wait_ld();
                    if (h == 1) {
                        fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(s_free);   // the producer may overwrite S^T / dP^T
                    }
                    const bool tail = half_tail && i == n - 1;   // the sub-tile that ends at S
                    if (i == 0) {
                        if (tail) compute(Masked{}, Masked{}, h, sr, dr);
                        else compute(Masked{}, Plain{}, h, sr, dr);
                    } else {
                        if (tail) compute(Plain{}, Masked{}, h, sr, dr);
                        else compute(Plain{}, Plain{}, h, sr, dr);
                    }
                }
                // dS^T was last read by dK / dQ of the previous sub-tile, P^T by its dV
                ok = g == 0 || mbar_wait(ds_free, (g - 1) & 1, abort_flag);
                if (!__all_sync(0xffffffffu, ok)) {
                    ok = false;
                    break;
                }
                // dS^T row r, queries c0 .. c0 + 31: atom c0 / 64, 16-byte chunks (c0 % 64) / 8 .. +3
                const uint32_t drow = sdS + (uint32_t)(c0 >> 6) * PA_BYTES + (uint32_t)r * 128u;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint32_t sw = (uint32_t)(((((c0 & 63) >> 3) + c) ^ (r & 7)) << 4);
                    st_shared_v4(drow + sw, dk[4 * c], dk[4 * c + 1], dk[4 * c + 2], dk[4 * c + 3]);
                }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive(ds_full);
                ok = g == 0 || mbar_wait(p_free, (g - 1) & 1, abort_flag);
                if (!__all_sync(0xffffffffu, ok)) {
                    ok = false;
                    break;
                }
                fence_after();
                tmem_st16(tmem + lane_off + P_COL + (uint32_t)(cg * 16), pk);
                tmem_wait_st();
                fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(p_full);
                    mbar_arrive(q_empty(s));
                }
            }
        }
    } else {
        // ------------------------------------------- dQ drain, dK / dV out ----
        const int lg = warp & 3;
        const int r = lg * 32 + lane;                         // query row of the sub-tile / key row of the item
        const uint32_t lane_off = (uint32_t)(lg * 32) << 16;
        const bool elected = warp == WD && lane == 0;
        int g = 0;
        bool ok = true;
        for (int t = 0, u = blockIdx.x; u < num_items; ++t, u += gridDim.x) {
            const Item it = item_of(u, BH, H, S);
            const int n = subtiles(u);
            for (int i = 0; i < n; ++i, ++g) {
                ok = __all_sync(0xffffffffu, ok && mbar_wait(dq_full, g & 1, abort_flag));
                if (ok) fence_after();
#pragma unroll 1
                for (int hc = 0; hc < 2; ++hc) {              // 32 columns at a time through the staging tile
                    uint32_t a[32];
                    if (ok) {
                        tmem_ld32(tmem + lane_off + DQ_COL + hc * 32, a);
                        tmem_wait_ld();
                        if (hc == 1) {
                            fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(dq_free);
                        }
                    }
                    if (elected) bulk_wait_read0();           // the previous reduce-add has read the staging
                    named_sync(1, 128);
                    if (ok) {
#pragma unroll
                        for (int c = 0; c < 8; ++c)
                            st_shared_v4(stage_addr(sStg, r, c), __float_as_uint(__uint_as_float(a[4 * c]) * scale),
                                         __float_as_uint(__uint_as_float(a[4 * c + 1]) * scale),
                                         __float_as_uint(__uint_as_float(a[4 * c + 2]) * scale),
                                         __float_as_uint(__uint_as_float(a[4 * c + 3]) * scale));
                    }
                    fence_proxy_async();
                    named_sync(1, 128);
                    // query block kb + i (128 rows) is entry 2 (kb + i) of the item's 64-row counters
                    int* sem = dq_sem ? dq_sem + (size_t)it.bh * (S / 64) + 2 * (it.kb + i) : nullptr;
                    if (elected && ok && sem && hc == 0) {
                        ok = wait_count(sem, it.kb, abort_flag);   // key blocks 0 .. kb-1 have added
                        fence_proxy_async_global();
                    }
                    if (elected && ok) {
                        // the sub-tile that ends at a half block adds only its 64 rows inside the sequence
                        const bool tail = half_tail && i == n - 1;
                        tma_reduce_add_2d(tail ? &tmdq64 : &tmdq, sStg, it.h * HD + hc * 32, it.krow0 + i * BQ);
                        bulk_commit();
                        if (sem && hc == 1) {                      // both halves complete: count this one
                            bulk_wait0();
                            fence_proxy_async_global();
                            __threadfence();
                            atomicAdd(sem, 1);
                        }
                    }
                }
            }
            // dK (scaled) and dV: TMEM -> FP16 in the item's K / V tiles (128B-swizzled rows, the
            // layout the TMA store reads), then the accumulators are free for the next item
            ok = __all_sync(0xffffffffu, ok && mbar_wait(acc_done, t & 1, abort_flag));
            const int kvb = t & 1;
            if (ok) {
                fence_after();
#pragma unroll 1
                for (int q = 0; q < 4; ++q) {                 // dK lo, dK hi, dV lo, dV hi
                    const int tv = q >> 1, hc = q & 1;
                    uint32_t a[32];
                    tmem_ld32(tmem + lane_off + (tv ? DV_COL : DK_COL) + hc * 32, a);
                    tmem_wait_ld();
                    const float f = tv ? 1.0f : scale;
                    const uint32_t row = (tv ? sV(kvb) : sK(kvb)) + (uint32_t)r * 128u;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        uint32_t w[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            w[e] = pack_h2(__uint_as_float(a[8 * c + 2 * e]) * f, __uint_as_float(a[8 * c + 2 * e + 1]) * f);
                        st_shared_v4(row + (uint32_t)((((hc * 4 + c) ^ (r & 7))) << 4), w[0], w[1], w[2], w[3]);
                    }
                }
                fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(acc_free);         // the next item may accumulate again
            }
            fence_proxy_async();
            named_sync(1, 128);
            if (elected && ok) {
                // a half last key block stores its 64 rows inside the sequence only
                const CUtensorMap* to = (half_tail && it.kb == nkb - 1) ? &tmout64 : &tmout;
                tma_store_2d(to, sK(kvb), D + it.h * HD, it.krow0);
                tma_store_2d(to, sV(kvb), 2 * D + it.h * HD, it.krow0);
                bulk_commit();
                bulk_wait_read0();                            // tiles read: the buffer may take new K / V
                mbar_arrive(kv_empty(kvb));
            }
        }
        if (elected) bulk_wait0();
    }
    fence_before();
    __syncthreads();
    fence_after();
    if (threadIdx.x == 0 && *abort_flag) atomicExch(err, RBK_ERR_TIMEOUT);
    if (warp == 1) tmem_free(tmem, TMEM_COLS);
}

}  // namespace attn_tc_bwd

// ---------------------------------------------------------------------------
// d_head 128.  The same work items and P / dS computation, but the d_head-64
// TMEM map does not fit: dK and dV alone take 256 of the 512 columns.  So
//   * S^T and dP^T are single-buffered (64 + 64 columns); the P / dS warps free
//     them as soon as they have loaded them, and the consumer-side MMAs of the
//     previous sub-tile keep the tensor pipe busy meanwhile;
//   * dQ is produced transposed per 64-query sub-tile,
//       dQ^T_i = K^T dS^T_i   (M = 128 = d_head, N = 64 queries, K = 128 keys),
//     with K read MN-major and dS^T_i as the MN-major B operand: 64 columns;
//   * P^T stays double-buffered in TMEM (2 x 32 columns of FP16 pairs).
// TMEM: S^T 0, dP^T 64, P^T[2] 128/160, dQ^T 192, dK 256, dV 384.
// Shared memory (one CTA per SM): K, V (single-buffered, 32 KB each), Q / dO
// ring of 4 (16 KB each), dS^T[2] (16 KB each), the per-query rows.  The drain
// warps hold one d_head column of dQ^T per thread and add it into the FP32
// accumulator with red.global (a warp covers 32 consecutive columns of one
// query row: one 128-byte line per instruction); dK and dV leave straight from
// registers, one key row per thread.
namespace attn_tc_bwd128 {

using namespace tc;
using attn_tc_bwd::ex2;
using attn_tc_bwd::pack_h2;
using attn_tc_bwd::st_shared_v4;
using attn_tc_bwd::ld_shared_f4;
using attn_tc_bwd::Item;
using attn_tc_bwd::ld_acquire;
using attn_tc_bwd::wait_count;
using attn_tc_bwd::item_of;
using attn_tc_bwd::Masked;
using attn_tc_bwd::Plain;

constexpr int BK = 128, BQ = 64, HD = 128;
constexpr int QS = 4;                       // Q / dO ring depth
constexpr int NE = 16;                      // P / dS warps
constexpr int WE = 3;                       // first P / dS warp
constexpr int WD = WE + NE;                 // first drain warp
constexpr int kThreads = (WD + 4) * 32;
constexpr int KT_BYTES = BK * HD * 2;       // 32 KB  K or V block (two 64-column atoms of 16 KB)
constexpr int KA_BYTES = BK * 128;          // one atom of K / V
constexpr int QT_BYTES = BQ * HD * 2;       // 16 KB  Q or dO sub-tile (two atoms of 8 KB)
constexpr int QA_BYTES = BQ * 128;
constexpr int PT_BYTES = BK * BQ * 2;       // 16 KB  dS^T sub-tile
constexpr int ROW_BYTES = 2 * BQ * 4;       // -LSE log2e | Dot of one sub-tile
constexpr int OFF_K = 0, OFF_V = OFF_K + KT_BYTES, OFF_Q = OFF_V + KT_BYTES, OFF_DO = OFF_Q + QS * QT_BYTES,
              OFF_DS = OFF_DO + QS * QT_BYTES, OFF_ROW = OFF_DS + 2 * PT_BYTES, OFF_BAR = OFF_ROW + QS * ROW_BYTES;
constexpr int NBARS = 2 * QS + 2 + 2 + 2 * 2 + 2 + 2;
constexpr int SMEM_USED = OFF_BAR + NBARS * 8 + 16;
constexpr int SMEM = 232448;                // the per-CTA maximum; the base must come 1024-aligned
static_assert(SMEM_USED <= SMEM, "shared memory budget");
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t S_COL = 0, DP_COL = 64, P_COL = 128, DQ_COL = 192, DK_COL = 256, DV_COL = 384;

__device__ __forceinline__ void red_add(float* p, float v) {
    asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    flash_bwd_tc128_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmkv,
                           const __grid_constant__ CUtensorMap tmdo, half* __restrict__ dqkv,
                           float* __restrict__ dq_acc, const float* __restrict__ NL2, const float* __restrict__ Dot,
                           int S, int H, int num_items, float scale, float scale_log2, int* err,
                           int* __restrict__ dq_sem) {
    extern __shared__ __align__(1024) uint8_t smem128[];
    const uint32_t raw = su32(smem128);
    const uint32_t base = (raw + 1023u) & ~1023u;
    if (base - raw + SMEM_USED > (uint32_t)SMEM) {   // uniform: no smem, TMEM or barrier touched yet
        if (threadIdx.x == 0) atomicExch(err, RBK_ERR_UNSUPPORTED);
        return;
    }
    uint8_t* gbase = smem128 + (base - raw);
    const uint32_t sK = base + OFF_K, sV = base + OFF_V;
    auto sQ = [&](int s) { return base + OFF_Q + (uint32_t)s * QT_BYTES; };
    auto sdO = [&](int s) { return base + OFF_DO + (uint32_t)s * QT_BYTES; };
    auto sRow = [&](int s) { return base + OFF_ROW + (uint32_t)s * ROW_BYTES; };
    auto sdS = [&](int s) { return base + OFF_DS + (uint32_t)s * PT_BYTES; };
    const uint32_t bars = base + OFF_BAR;
    auto q_full = [&](int s) { return bars + 8 * s; };
    auto q_empty = [&](int s) { return bars + 8 * QS + 8 * s; };
    const uint32_t b2 = bars + 16 * QS;
    const uint32_t kv_full = b2, kv_empty = b2 + 8;     // K, V of the item / released by both issuers
    const uint32_t s_full = b2 + 16, s_free = b2 + 24;  // S^T, dP^T in TMEM / loaded by the P / dS warps
    auto p_full = [&](int s) { return b2 + 32 + 8 * s; };   // P^T_i in TMEM, dS^T_i in shared memory
    auto p_free = [&](int s) { return b2 + 48 + 8 * s; };   // dV_i, dK_i, dQ^T_i done: buffers i & 1 reusable
    const uint32_t dq_full = b2 + 64, dq_free = b2 + 72, acc_done = b2 + 80, acc_free = b2 + 88;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_BAR + NBARS * 8);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + OFF_BAR + NBARS * 8 + 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int BH = num_items / ((S + BK - 1) / BK);
    const int D = H * HD;

    if (threadIdx.x == 0) {
        for (int s = 0; s < QS; ++s) {
            mbar_init(q_full(s), 1);
            mbar_init(q_empty(s), NE + 2);
        }
        mbar_init(kv_full, 1);
        mbar_init(kv_empty, 2);
        mbar_init(s_full, 1);
        mbar_init(s_free, NE);
        for (int s = 0; s < 2; ++s) {
            mbar_init(p_full(s), NE);
            mbar_init(p_free(s), 1);
        }
        mbar_init(dq_full, 1);
        mbar_init(dq_free, 4);
        mbar_init(acc_done, 1);
        mbar_init(acc_free, 4);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0 && lane == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmq) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmkv) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmdo) : "memory");
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_dependency_sync();

    if (warp == 0) {
        // ---------------------------------------------------------- TMA ----
        if (lane == 0) {
            int g = 0;
            bool ok = true;
            for (int t = 0, u = blockIdx.x; ok && u < num_items; ++t, u += gridDim.x) {
                const Item it = item_of(u, BH, H, S);
                if (!mbar_wait(kv_empty, (t & 1) ^ 1, abort_flag)) break;
                mbar_expect_tx(kv_full, 2 * KT_BYTES);
#pragma unroll
                for (int a = 0; a < 2; ++a) {
                    tma_load_2d(sK + a * KA_BYTES, &tmkv, kv_full, D + it.h * HD + 64 * a, it.krow0);
                    tma_load_2d(sV + a * KA_BYTES, &tmkv, kv_full, 2 * D + it.h * HD + 64 * a, it.krow0);
                }
                const float* nl2 = NL2 + (size_t)it.bh * S + it.kb * BK;
                const float* dot = Dot + (size_t)it.bh * S + it.kb * BK;
                for (int i = 0; i < it.n; ++i, ++g) {
                    const int s = g % QS;
                    if (!mbar_wait(q_empty(s), ((g / QS) & 1) ^ 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = q_full(s);
                    mbar_expect_tx(fb, 2 * QT_BYTES + ROW_BYTES);
#pragma unroll
                    for (int a = 0; a < 2; ++a) {
                        tma_load_2d(sQ(s) + a * QA_BYTES, &tmq, fb, it.h * HD + 64 * a, it.krow0 + i * BQ);
                        tma_load_2d(sdO(s) + a * QA_BYTES, &tmdo, fb, it.h * HD + 64 * a, it.krow0 + i * BQ);
                    }
                    bulk_load(sRow(s), nl2 + i * BQ, BQ * 4, fb);
                    bulk_load(sRow(s) + BQ * 4, dot + i * BQ, BQ * 4, fb);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------- MMA: S^T, dP^T producer ----
        if (lane == 0) {
            const uint32_t id_s = idesc_f16(BQ, 0, 0);    // K (K-major) x Q^T (K-major): N = 64 queries
            int g = 0;
            bool ok = true;
            for (int t = 0, u = blockIdx.x; ok && u < num_items; ++t, u += gridDim.x) {
                const int n = item_of(u, BH, H, S).n;
                if (!mbar_wait(kv_full, t & 1, abort_flag)) break;
                for (int i = 0; i < n; ++i, ++g) {
                    const int s = g % QS;
                    ok = mbar_wait(q_full(s), (g / QS) & 1, abort_flag) &&
                         (g == 0 || mbar_wait(s_free, (g - 1) & 1, abort_flag));
                    if (!ok) break;
                    fence_after();
#pragma unroll
                    for (int k = 0; k < HD / 16; ++k)
                        mma_f16(tmem + S_COL, sdesc(sK + (k >> 2) * KA_BYTES + (k & 3) * 32, 16, 1024),
                                sdesc(sQ(s) + (k >> 2) * QA_BYTES + (k & 3) * 32, 16, 1024), id_s, k > 0);
#pragma unroll
                    for (int k = 0; k < HD / 16; ++k)
                        mma_f16(tmem + DP_COL, sdesc(sV + (k >> 2) * KA_BYTES + (k & 3) * 32, 16, 1024),
                                sdesc(sdO(s) + (k >> 2) * QA_BYTES + (k & 3) * 32, 16, 1024), id_s, k > 0);
                    mma_commit(s_full);
                    mma_commit(q_empty(s));
                }
                if (ok) mma_commit(kv_empty);
            }
        }
    } else if (warp == 2) {
        // ------------------------------------------- MMA: dQ^T, dV, dK consumer ----
        if (lane == 0) {
            const uint32_t id_kv = idesc_f16(HD, 0, 1);   // P^T (TMEM) / dS^T (K-major) x dO / Q (MN-major): N = 128
            const uint32_t id_q = idesc_f16(BQ, 1, 1);    // K^T (MN-major) x dS^T (MN-major): N = 64 queries
            int g = 0;
            bool ok = true;
            for (int t = 0, u = blockIdx.x; ok && u < num_items; ++t, u += gridDim.x) {
                const int n = item_of(u, BH, H, S).n;
                // K is an operand of dQ^T; the accumulators must have been read out for the previous item
                ok = mbar_wait(kv_full, t & 1, abort_flag) && (t == 0 || mbar_wait(acc_free, (t - 1) & 1, abort_flag));
                if (!ok) break;
                for (int i = 0; i < n; ++i, ++g) {
                    const int s = g % QS, pb = g & 1;
                    ok = mbar_wait(p_full(pb), (g >> 1) & 1, abort_flag) &&
                         (g == 0 || mbar_wait(dq_free, (g - 1) & 1, abort_flag));   // dQ^T_{g-1} read out
                    if (!ok) break;
                    fence_after();
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        mma_f16(tmem + DQ_COL, sdesc(sK + k * 2048, KA_BYTES, 1024), sdesc(sdS(pb) + k * 2048, PT_BYTES, 1024),
                                id_q, k > 0);
                    mma_commit(dq_full);
#pragma unroll
                    for (int k = 0; k < BQ / 16; ++k)
                        mma_f16_ts(tmem + DV_COL, tmem + P_COL + (uint32_t)(pb * 32 + k * 8),
                                   sdesc(sdO(s) + k * 2048, QA_BYTES, 1024), id_kv, (i > 0 || k > 0) ? 1u : 0u);
#pragma unroll
                    for (int k = 0; k < BQ / 16; ++k)
                        mma_f16(tmem + DK_COL, sdesc(sdS(pb) + k * 32, 16, 1024), sdesc(sQ(s) + k * 2048, QA_BYTES, 1024),
                                id_kv, (i > 0 || k > 0) ? 1u : 0u);
                    mma_commit(q_empty(s));
                    mma_commit(p_free(pb));
                }
                if (ok) {
                    mma_commit(acc_done);
                    mma_commit(kv_empty);
                }
            }
        }
    } else if (warp < WD) {
        // ------------------------------------------------------ P / dS ----
        const int lg = warp & 3, quarter = (warp - WE) >> 2;
        const int r = lg * 32 + lane;                         // key row inside the block
        const uint32_t lane_off = (uint32_t)(lg * 32) << 16;
        const int c0 = quarter * 16;                          // first query column of this warp
        int g = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < num_items; u += gridDim.x) {
            const int n = item_of(u, BH, H, S).n;
            for (int i = 0; i < n; ++i, ++g) {
                const int s = g % QS, pb = g & 1;
                ok = mbar_wait(s_full, g & 1, abort_flag) && mbar_wait(q_full(s), (g / QS) & 1, abort_flag);
                if (!__all_sync(0xffffffffu, ok)) {
                    ok = false;
                    break;
                }
                fence_after();
                uint32_t sr[16], dr[16];
                tmem_ld16(tmem + lane_off + S_COL + c0, sr);
                tmem_ld16(tmem + lane_off + DP_COL + c0, dr);
                tmem_wait_ld();
                fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(s_free);           // the producer may compute the next sub-tile
                const uint32_t rowp = sRow(s);
                const uint64_t c2 = pair_of(scale_log2);
                uint32_t pk[8], dk[8];
                auto compute = [&](auto masked) {
                    const int lim = r - BQ * i - c0;
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const float4 nl = ld_shared_f4(rowp + (uint32_t)(c0 + 4 * q4) * 4);
                        const float4 dt = ld_shared_f4(rowp + BQ * 4 + (uint32_t)(c0 + 4 * q4) * 4);
                        const float nlv[4] = {nl.x, nl.y, nl.z, nl.w}, dtv[4] = {dt.x, dt.y, dt.z, dt.w};
                        float pv[4], dv[4];
#pragma unroll
                        for (int e4 = 0; e4 < 4; e4 += 2) {       // packed FP32 pairs
                            const int e = 4 * q4 + e4;
                            float x0, x1;
                            ffma2v(x0, x1, __uint_as_float(sr[e]), __uint_as_float(sr[e + 1]), c2, nlv[e4],
                                   nlv[e4 + 1]);
                            float p0 = ex2(x0), p1 = ex2(x1);
                            if (decltype(masked)::value) {
                                p0 = e < lim ? 0.0f : p0;
                                p1 = e + 1 < lim ? 0.0f : p1;
                            }
                            pv[e4] = p0;
                            pv[e4 + 1] = p1;
                            float d0, d1;
                            fsub2(d0, d1, __uint_as_float(dr[e]), __uint_as_float(dr[e + 1]), dtv[e4], dtv[e4 + 1]);
                            fmul2(dv[e4], dv[e4 + 1], p0, p1, d0, d1);
                        }
                        pk[2 * q4] = pack_h2(pv[0], pv[1]);
                        pk[2 * q4 + 1] = pack_h2(pv[2], pv[3]);
                        dk[2 * q4] = pack_h2(dv[0], dv[1]);
                        dk[2 * q4 + 1] = pack_h2(dv[2], dv[3]);
                    }
                };
                if (i < 2) compute(Masked{});
                else compute(Plain{});
                // P^T buffer pb and dS^T buffer pb were last read by the MMAs of sub-tile g - 2
                ok = g < 2 || mbar_wait(p_free(pb), ((g >> 1) & 1) ^ 1, abort_flag);
                if (!__all_sync(0xffffffffu, ok)) {
                    ok = false;
                    break;
                }
                fence_after();
                tmem_st8(tmem + lane_off + P_COL + (uint32_t)(pb * 32 + quarter * 8), pk);
                const uint32_t drow = sdS(pb) + (uint32_t)r * 128u;
#pragma unroll
                for (int c = 0; c < 2; ++c) {                 // 16-byte chunk = 8 queries, 128B swizzle
                    const uint32_t sw = (uint32_t)((((c0 >> 3) + c) ^ (r & 7)) << 4);
                    st_shared_v4(drow + sw, dk[4 * c], dk[4 * c + 1], dk[4 * c + 2], dk[4 * c + 3]);
                }
                tmem_wait_st();
                fence_proxy_async();
                fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(p_full(pb));
                    mbar_arrive(q_empty(s));
                }
            }
        }
    } else {
        // ------------------------------------------- dQ drain, dK / dV out ----
        const int lg = warp & 3;
        const int r = lg * 32 + lane;                         // d_head column of dQ^T / key row of the item
        const uint32_t lane_off = (uint32_t)(lg * 32) << 16;
        int g = 0;
        bool ok = true;
        for (int t = 0, u = blockIdx.x; ok && u < num_items; ++t, u += gridDim.x) {
            const Item it = item_of(u, BH, H, S);
            for (int i = 0; i < it.n; ++i, ++g) {
                ok = __all_sync(0xffffffffu, mbar_wait(dq_full, g & 1, abort_flag));
                if (!ok) break;
                fence_after();
                // deterministic dQ: 64-query block 2 kb + i takes the key blocks in ascending order; each
                // of the 4 drain warps counts its own part, so key block kb waits for 4 kb arrivals
                int* sem = dq_sem ? dq_sem + (size_t)it.bh * (S / 64) + 2 * it.kb + i : nullptr;
                if (sem) {
                    bool w = true;
                    if (lane == 0) w = wait_count(sem, 4 * it.kb, abort_flag);
                    ok = __shfl_sync(0xffffffffu, w, 0);
                    if (!ok) break;
                    (void)ld_acquire(sem);                    // every lane orders its adds after the count
                }
                float* dst = dq_acc + (size_t)(it.krow0 + i * BQ) * D + it.h * HD + r;
#pragma unroll 1
                for (int hc = 0; hc < 2; ++hc) {              // 32 queries at a time
                    uint32_t a[32];
                    tmem_ld32(tmem + lane_off + DQ_COL + hc * 32, a);
                    tmem_wait_ld();
                    if (hc == 1) {
                        fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(dq_free);
                    }
#pragma unroll
                    for (int c = 0; c < 32; ++c) red_add(dst + (size_t)(hc * 32 + c) * D, __uint_as_float(a[c]) * scale);
                }
                if (sem) {
                    __threadfence();
                    __syncwarp();
                    if (lane == 0) {
                        __threadfence();
                        atomicAdd(sem, 1);
                    }
                }
            }
            if (!ok) break;
            // dK (scaled) and dV: TMEM -> FP16 -> global, one key row per thread
            ok = __all_sync(0xffffffffu, mbar_wait(acc_done, t & 1, abort_flag));
            if (!ok) break;
            fence_after();
            half* krow = dqkv + (size_t)(it.krow0 + r) * 3 * D + D + it.h * HD;
#pragma unroll 1
            for (int q = 0; q < 8; ++q) {                     // dK in 4 x 32 columns, then dV
                const int tv = q >> 2, hc = q & 3;
                uint32_t a[32];
                tmem_ld32(tmem + lane_off + (tv ? DV_COL : DK_COL) + hc * 32, a);
                tmem_wait_ld();
                if (q == 7) {
                    fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(acc_free);     // the next item may accumulate again
                }
                const float f = tv ? 1.0f : scale;
                uint4* out = reinterpret_cast<uint4*>(krow + tv * D + hc * 32);
                const bool inside = it.kb * BK + r < S;       // key rows of a half last block beyond S: none
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint4 w;
                    w.x = pack_h2(__uint_as_float(a[8 * c + 0]) * f, __uint_as_float(a[8 * c + 1]) * f);
                    w.y = pack_h2(__uint_as_float(a[8 * c + 2]) * f, __uint_as_float(a[8 * c + 3]) * f);
                    w.z = pack_h2(__uint_as_float(a[8 * c + 4]) * f, __uint_as_float(a[8 * c + 5]) * f);
                    w.w = pack_h2(__uint_as_float(a[8 * c + 6]) * f, __uint_as_float(a[8 * c + 7]) * f);
                    if (inside) out[c] = w;
                }
            }
        }
    }
    fence_before();
    __syncthreads();
    fence_after();
    if (threadIdx.x == 0 && *abort_flag) atomicExch(err, RBK_ERR_TIMEOUT);
    if (warp == 1) tmem_free(tmem, TMEM_COLS);
}

}  // namespace attn_tc_bwd128

// Main pass of rbk_attn_bwd (attn.cu) for d_head 64 or 128 and S % 64 == 0 (a sequence that ends in
// a half 128-row block: the tail sub-tile masks its queries beyond S, and the stores and dQ
// additions of the last blocks cover only their rows inside the sequence).
// dq_acc: FP32 [B*S, H*dh], zeroed; NL2 / Dot: [B*H, S].  Writes the k and v
// sections of dqkv and adds dQ into dq_acc.
int attn_bwd_tc(rbk_ctx* ctx, void* dqkv, float* dq_acc, const void* qkv, const void* dout, const float* NL2,
                const float* Dot, int B, int S, int H, int dh, float scale, cudaStream_t st, int* dq_sem) {
    const uint64_t BS = (uint64_t)B * S;
    const int items = B * H * ((S + 127) / 128);
    const int grid = items < ctx->num_sms ? items : ctx->num_sms;
    if (dh == 128) {
        using namespace attn_tc_bwd128;
        const int D = H * HD;
        CUtensorMap tmq, tmkv, tmdo;
        RBK_TRY(tc::make_tmap(&tmq, qkv, 3 * (uint64_t)D, BS, 3 * (uint64_t)D, 64, BQ));
        RBK_TRY(tc::make_tmap(&tmkv, qkv, 3 * (uint64_t)D, BS, 3 * (uint64_t)D, 64, BK));
        RBK_TRY(tc::make_tmap(&tmdo, dout, (uint64_t)D, BS, (uint64_t)D, 64, BQ));
        static int set_dev = -1;
        if (set_dev != ctx->device) {
            RBK_CUDA(cudaFuncSetAttribute(flash_bwd_tc128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
            set_dev = ctx->device;
        }
        RBK_CUDA(launch_pdl(flash_bwd_tc128_kernel, dim3(grid), dim3(kThreads), SMEM, st, tmq, tmkv, tmdo, (half*)dqkv,
                            dq_acc, NL2, Dot, S, H, items, scale, scale * 1.4426950408889634f,
                            ctx->tickets + kGemmError, dq_sem));
        RBK_LAUNCHED("flash_bwd_tc128_kernel");
        return RBK_OK;
    }
    if (dh != 64) return RBK_ERR_UNSUPPORTED;
    using namespace attn_tc_bwd;
    const int D = H * HD;
    CUtensorMap tmq, tmkv, tmdo, tmdq, tmout, tmdq64, tmout64;
    RBK_TRY(tc::make_tmap(&tmq, qkv, 3 * (uint64_t)D, BS, 3 * (uint64_t)D, 64, BQ));
    RBK_TRY(tc::make_tmap(&tmkv, qkv, 3 * (uint64_t)D, BS, 3 * (uint64_t)D, 64, BK));
    RBK_TRY(tc::make_tmap(&tmdo, dout, (uint64_t)D, BS, (uint64_t)D, 64, BQ));
    RBK_TRY(tc::make_tmap(&tmdq, dq_acc, (uint64_t)D, BS, (uint64_t)D, 32, 128, CU_TENSOR_MAP_DATA_TYPE_FLOAT32));
    RBK_TRY(tc::make_tmap(&tmout, dqkv, 3 * (uint64_t)D, BS, 3 * (uint64_t)D, 64, BK));
    // the 64 rows of a half last block (sequences of 128 k + 64)
    RBK_TRY(tc::make_tmap(&tmdq64, dq_acc, (uint64_t)D, BS, (uint64_t)D, 32, 64, CU_TENSOR_MAP_DATA_TYPE_FLOAT32));
    RBK_TRY(tc::make_tmap(&tmout64, dqkv, 3 * (uint64_t)D, BS, 3 * (uint64_t)D, 64, 64));
    static int set_dev = -1;
    if (set_dev != ctx->device) {
        RBK_CUDA(cudaFuncSetAttribute(flash_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        set_dev = ctx->device;
    }
    RBK_CUDA(launch_pdl(flash_bwd_tc_kernel, dim3(grid), dim3(kThreads), SMEM, st, tmq, tmkv, tmdo, tmdq, tmout, NL2,
                        Dot, S, H, items, scale, scale * 1.4426950408889634f, ctx->tickets + kGemmError, dq_sem,
                        tmdq64, tmout64));
    RBK_LAUNCHED("flash_bwd_tc_kernel");
    return RBK_OK;
}

}  // namespace rbk
