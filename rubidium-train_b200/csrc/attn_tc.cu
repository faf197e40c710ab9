// attn_tc.cu — causal flash attention forward on the 5th-generation tensor
// cores (d_head 64 or 128): the tcgen05 replacement of the mma.sync forward in
// attn.cu for sequence lengths that are multiples of 128.
//
// Persistent CTAs (two per SM at d_head 64, one at 128) take tiles = (batch,
// head, 128-query block) from a device counter, longest query blocks first
// within groups of heads; the TMA lane loads the next tile's Q and K/V while
// the softmax warps finish the current tile's epilogue, and every role learns
// the tile sequence through a two-slot ring in shared memory.  (One CTA per
// tile, 5 waves at GPT-2-small shapes, took 72.7 us against 63.7 us at d_head
// 64.)  Keys are consumed 64 at a time.  Q and K tiles are d_head/64 128B-swizzle
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
// Sequence lengths that are 64 more than a multiple of 128 end in a half query
// block: its Q rows beyond the sequence are the next sequence's (or TMA's zero
// fill after the last), computed but never stored; the keys beyond the
// sequence are above every stored query, so the causal mask zeroes them.
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
    static constexpr int SMEM = 1024 + OFF_BAR + 512;
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
// Tile t of the persistent schedule -> (query block, batch*head).  Heads are
// taken in groups of hpg; inside a group the longest query blocks (most keys
// under the causal mask) come first, all heads of the group at each length.
// Group-wise keeps one group's K/V in L2 while the longest-first order inside
// it balances the CTAs, which take tiles from a device counter as they finish.
__device__ __forceinline__ void fwd_tile(int t, int nqb, int BH, int hpg, int& qb, int& bh) {
    const int per = hpg * nqb;
    const int g = t / per, r = t - g * per;
    const int h0 = g * hpg;
    const int hg = BH - h0 < hpg ? BH - h0 : hpg;
    qb = nqb - 1 - r / hg;
    bh = h0 + r % hg;
}

template <int HD>
__global__ void __launch_bounds__(FwdCfg<HD>::THREADS, FwdCfg<HD>::CTAS_PER_SM)
    flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmkv, half* O,
                        float* LSE, int S, int H, int BH, int hpg, float scale_log2, int* tile_ctr, int* err) {
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
    // barriers: q_full | q_empty | k_full[KS] | k_empty[KS] | v_full[VS] | v_empty[VS] | s_full[2] | p_full[2] |
    // o_done[2] | o_free | t_full[2] | t_empty[2] | ml_full | ml_read (one barrier per buffer, so a wait never
    // targets a phase two completions old)
    const uint32_t bars = base + OFF_BAR;
    const uint32_t q_full = bars, q_empty = bars + 8;
    auto k_full = [&](int s) { return bars + 16 + 8 * s; };
    auto k_empty = [&](int s) { return bars + 16 + 8 * KS + 8 * s; };
    auto v_full = [&](int s) { return bars + 16 + 16 * KS + 8 * s; };
    auto v_empty = [&](int s) { return bars + 16 + 16 * KS + 8 * VS + 8 * s; };
    const uint32_t bars2 = bars + 16 + 16 * KS + 16 * VS;
    auto s_full = [&](int s) { return bars2 + 8 * s; };
    auto p_full = [&](int s) { return bars2 + 16 + 8 * s; };
    auto o_done = [&](int s) { return bars2 + 32 + 8 * s; };
    const uint32_t o_free = bars2 + 48;
    auto t_full = [&](int s) { return bars2 + 56 + 8 * s; };
    auto t_empty = [&](int s) { return bars2 + 72 + 8 * s; };
    const uint32_t ml_full = bars2 + 88, ml_read = bars2 + 96;   // two-group (m, l) exchange
    uint8_t* misc = gbase + (bars2 - base) + 104;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 4);
    volatile int* tile_slot = reinterpret_cast<volatile int*>(misc + 8);   // [2]: the tile ring

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nqb = (S + BQ - 1) / BQ;
    const int ntiles = nqb * BH;
    const int D = H * HD;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int s = 0; s < KS; ++s) { mbar_init(k_full(s), 1); mbar_init(k_empty(s), 1); }
        for (int s = 0; s < VS; ++s) { mbar_init(v_full(s), 1); mbar_init(v_empty(s), 1); }
        mbar_init(s_full(0), 1); mbar_init(s_full(1), 1);
        for (int s = 0; s < 2; ++s) { mbar_init(p_full(s), 4); mbar_init(o_done(s), 1); }
        mbar_init(o_free, 4 * NG);                    // every softmax warp has read O out of TMEM
        for (int s = 0; s < 2; ++s) {
            mbar_init(t_full(s), 1);
            mbar_init(t_empty(s), 2 + 4 * NG);        // V lane, MMA lane, softmax warps
        }
        mbar_init(ml_full, 4 * NG);
        mbar_init(ml_read, 4 * NG);
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

    // Every role walks the same tile sequence: lane 0 of warp 0 takes tiles from the device
    // counter and publishes each through the two-slot tile ring; a tile index >= ntiles ends the
    // walk.  Key blocks, K/V ring positions and S/P/O buffer phases run on across tiles (every
    // tile has an even number of 64-key blocks, so buffer j & 1 of a tile is the running one).
    auto next_tile = [&](int tc) -> int {           // consumers: wait for tile tc (-1 on a timeout)
        const int slot = tc & 1;
        if (!mbar_wait(t_full(slot), (tc >> 1) & 1, abort_flag)) return -1;
        return tile_slot[slot];
    };

    if (warp == 0) {
        // ---------------------------------------------------------- TMA ----
        // lane 0 schedules tiles and streams Q then K, lane 16 streams V: the two rings refill
        // independently and run ahead into the next tile
        if (lane == 0) {
            int kc = 0;
            for (int tc = 0;; ++tc) {
                const int slot = tc & 1;
                if (!mbar_wait(t_empty(slot), ((tc >> 1) & 1) ^ 1, abort_flag)) break;
                const int t = atomicAdd(tile_ctr, 1);
                tile_slot[slot] = t;
                mbar_arrive(t_full(slot));
                if (t >= ntiles) break;
                int qb, bh;
                fwd_tile(t, nqb, BH, hpg, qb, bh);
                const int h = bh % H, row0 = (bh / H) * S, nkv = (qb + 1) * (BQ / BKV);
                if (!mbar_wait(q_empty, (tc & 1) ^ 1, abort_flag)) break;   // last S MMA of tile tc-1
                mbar_expect_tx(q_full, Q_BYTES);
#pragma unroll
                for (int a = 0; a < NA; ++a)
                    tma_load_2d(sQ + a * (BQ * 128), &tmq, q_full, h * HD + 64 * a, row0 + qb * BQ);
                bool ok = true;
                for (int j = 0; j < nkv; ++j, ++kc) {
                    const int ks = kc % KS;
                    if (!mbar_wait(k_empty(ks), ((kc / KS) & 1) ^ 1, abort_flag)) { ok = false; break; }
                    mbar_expect_tx(k_full(ks), KV_BYTES);
#pragma unroll
                    for (int a = 0; a < NA; ++a)
                        tma_load_2d(sK(ks) + a * (BKV * 128), &tmkv, k_full(ks), D + h * HD + 64 * a, row0 + j * BKV);
                }
                if (!ok) break;
            }
            // each CTA signs off once; the last one re-arms the counter for the next launch
            __threadfence();
            if (atomicAdd(tile_ctr + 1, 1) == (int)gridDim.x - 1) {
                atomicExch(tile_ctr, 0);
                atomicExch(tile_ctr + 1, 0);
            }
        } else if (lane == 16) {
            int vc = 0;
            for (int tc = 0;; ++tc) {
                const int t = next_tile(tc);
                if (t < 0) break;
                mbar_arrive(t_empty(tc & 1));
                if (t >= ntiles) break;
                int qb, bh;
                fwd_tile(t, nqb, BH, hpg, qb, bh);
                const int h = bh % H, row0 = (bh / H) * S, nkv = (qb + 1) * (BQ / BKV);
                bool ok = true;
                for (int j = 0; j < nkv; ++j, ++vc) {
                    const int vs = vc % VS;
                    if (!mbar_wait(v_empty(vs), ((vc / VS) & 1) ^ 1, abort_flag)) { ok = false; break; }
                    mbar_expect_tx(v_full(vs), KV_BYTES);
#pragma unroll
                    for (int a = 0; a < NA; ++a)
                        tma_load_2d(sV(vs) + a * (BKV * 128), &tmkv, v_full(vs), 2 * D + h * HD + 64 * a,
                                    row0 + j * BKV);
                }
                if (!ok) break;
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA ----
        if (lane == 0) {
            const uint32_t idesc_s = idesc_f16(BKV, 0, 0);   // Q (K-major) x K (K-major), N = 64
            const uint32_t idesc_o = idesc_f16(HD, 0, 1);    // P (K-major) x V (MN-major), N = d_head
            int kc = 0, vc = 0, jb = 0;                      // K / V ring positions, key blocks before this tile
            bool ok = true;
            for (int tc = 0; ok; ++tc) {
                const int t = next_tile(tc);
                if (t < 0) break;
                mbar_arrive(t_empty(tc & 1));
                if (t >= ntiles) break;
                int qb, bh;
                fwd_tile(t, nqb, BH, hpg, qb, bh);
                const int nkv = (qb + 1) * (BQ / BKV);
                auto issue_s = [&](int j) -> bool {
                    const int kk = kc + j;
                    const int ks = kk % KS;
                    if (!mbar_wait(k_full(ks), (kk / KS) & 1, abort_flag)) return false;
                    fence_after();
                    const uint32_t s_tm = tmem + (uint32_t)((jb + j) & 1) * BKV;
#pragma unroll
                    for (int k = 0; k < HD / 16; ++k)   // K = d_head: atom k / 4, 32 B per step inside it
                        mma_f16(s_tm, sdesc(sQ + (k >> 2) * (BQ * 128) + (k & 3) * 32, 16, 1024),
                                sdesc(sK(ks) + (k >> 2) * (BKV * 128) + (k & 3) * 32, 16, 1024), idesc_s, k > 0);
                    mma_commit(s_full((jb + j) & 1));
                    mma_commit(k_empty(ks));
                    if (j == nkv - 1) mma_commit(q_empty);    // the tile's last read of Q
                    return true;
                };
                // S of the first two blocks (nkv >= 2); O of the previous tile read out before PV
                ok = mbar_wait(q_full, tc & 1, abort_flag) && issue_s(0) && issue_s(1) &&
                     mbar_wait(o_free, (tc & 1) ^ 1, abort_flag);
                for (int j = 0; ok && j < nkv; ++j) {
                    const int J = jb + j;
                    const int vv = vc + j, vs = vv % VS;
                    if (!mbar_wait(p_full(J & 1), (J >> 1) & 1, abort_flag) ||
                        !mbar_wait(v_full(vs), (vv / VS) & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    fence_after();
                    const uint32_t o_tm = tmem + O_COL + (NG == 2 ? (uint32_t)(j & 1) * HD : 0u);   // the group's O
#pragma unroll
                    for (int k = 0; k < BKV / 16; ++k)
                        mma_f16(o_tm, sdesc(sP(J & 1) + k * 32, 16, 1024),
                                sdesc(sV(vs) + k * 2048, BKV * 128, 1024),   // N blocks of 64 columns, 8 KB apart
                                idesc_o, (j >= NG || k > 0) ? 1u : 0u);
                    mma_commit(o_done(J & 1));
                    mma_commit(v_empty(vs));
                    if (j + 2 < nkv && !issue_s(j + 2)) { ok = false; break; }   // S buffer released by p_full
                }
                kc += nkv;
                vc += nkv;
                jb += nkv;
            }
        }
    } else {
        // ------------------------------------------------------ softmax ----
        const int wg = NG == 2 ? (warp - 2) >> 2 : 0;    // two groups: even / odd key blocks
        const int q4 = warp & 3;
        const int row = q4 * 32 + lane;                   // query row inside the block
        const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
        const uint32_t o_col = O_COL + (uint32_t)wg * HD;
        bool ok = true;
        int jb = 0;
        for (int tc = 0; ok; ++tc) {
            const int t = next_tile(tc);
            if (t < 0) { ok = false; break; }
            __syncwarp();
            if (lane == 0) mbar_arrive(t_empty(tc & 1));
            if (t >= ntiles) break;
            int qb, bh;
            fwd_tile(t, nqb, BH, hpg, qb, bh);
            const int nkv = (qb + 1) * (BQ / BKV);
            const int qpos = qb * BQ + row;               // query position in the sequence
            float m = -INFINITY, l = 0.0f;                // running max (log2 units) and sum of this group
            int jl = 0;                                   // blocks of this group done
            for (int j = wg; j < nkv; j += NG, ++jl) {
                const int J = jb + j;
                const int sb = J & 1;                     // S / P buffer of block j
                if (!mbar_wait(s_full(sb), (J >> 1) & 1, abort_flag)) { ok = false; break; }
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
                    const int lim = qpos - j * BKV;       // keys e > lim are masked
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
                if (mx > m + 8.0f) {                      // lazy rescale (first block: m = -inf)
                    if (jl > 0) { corr = ex2(m - mx); rescale = true; }
                    m = mx;
                    l *= corr;
                }
                // P buffer sb (and, with two groups, O_wg) was last read by PV_{J-2}, possibly of the
                // previous tile
                if (J > 1) {
                    if (!mbar_wait(o_done(sb), ((J >> 1) & 1) ^ 1, abort_flag)) { ok = false; break; }
                    fence_after();
                }
                if (__any_sync(0xffffffffu, rescale)) {
                    if constexpr (NG == 1) {              // the single O must hold PV_{J-1} before its rescale
                        if (!mbar_wait(o_done((J - 1) & 1), ((J - 1) >> 1) & 1, abort_flag)) { ok = false; break; }
                        fence_after();
                    }
#pragma unroll 1
                    for (int c = 0; c < HD / 16; ++c) {
                        uint32_t tt[16];
                        tmem_ld16(tmem + lane_off + o_col + c * 16, tt);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 16; ++e) tt[e] = __float_as_uint(__uint_as_float(tt[e]) * corr);
                        tmem_st16(tmem + lane_off + o_col + c * 16, tt);
                    }
                    tmem_wait_st();
                }
                // p = 2^(s * scale * log2 e - m); a row with no visible key yet keeps m = -inf and p = 0.
                // Each 16-byte chunk of 8 keys goes to shared memory as soon as it is packed.
                const float nm = m == -INFINITY ? 0.0f : -m;
                const uint64_t c2 = pair_of(scale_log2), nm2 = pair_of(nm);
                uint64_t rs2[2] = {0, 0};                 // two packed (even, odd) sum accumulators
#pragma unroll
                for (int c = 0; c < 8; ++c) {             // 16-byte chunk = 8 keys, 128B swizzle
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
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pk[0]), "r"(pk[1]),
                                 "r"(pk[2]), "r"(pk[3])
                                 : "memory");
                }
                l += (__uint_as_float((uint32_t)rs2[0]) + __uint_as_float((uint32_t)(rs2[0] >> 32))) +
                     (__uint_as_float((uint32_t)rs2[1]) + __uint_as_float((uint32_t)(rs2[1] >> 32)));
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(p_full(sb));
            }
            if (!ok) break;
            // epilogue.  One group: O / l.  Two groups: after each has seen its last PV, swap (m, l)
            // and each writes half of the columns of
            // O = (O0 2^(m0-M) + O1 2^(m1-M)) / (l0 2^(m0-M) + l1 2^(m1-M)).
            const int jlast = jb + nkv - NG + wg;         // last block of this group (nkv is even)
            ok = mbar_wait(o_done(jlast & 1), (jlast >> 1) & 1, abort_flag);
            fence_after();
            float f0 = 0.0f, f1 = 0.0f, M = m, L = l;
            if constexpr (NG == 2) {
                // bounded mbarrier waits, not a named barrier: a group that leaves on a timeout must not
                // strand the other one
                float* ml = reinterpret_cast<float*>(gbase + Cf::OFF_ML);
                if (tc > 0) ok = ok && mbar_wait(ml_read, (tc - 1) & 1, abort_flag);   // tile tc-1's reads done
                ml[(wg * BQ + row) * 2] = m;
                ml[(wg * BQ + row) * 2 + 1] = l;
                __syncwarp();
                if (lane == 0) mbar_arrive(ml_full);
                ok = ok && mbar_wait(ml_full, tc & 1, abort_flag);
                const float m0 = ml[row * 2], l0 = ml[row * 2 + 1];
                const float m1 = ml[(BQ + row) * 2], l1 = ml[(BQ + row) * 2 + 1];
                __syncwarp();
                if (lane == 0) mbar_arrive(ml_read);
                M = fmaxf(m0, m1);
                const float a0 = m0 == -INFINITY ? 0.0f : ex2(m0 - M), a1 = m1 == -INFINITY ? 0.0f : ex2(m1 - M);
                L = l0 * a0 + l1 * a1;
                f0 = a0 / L;
                f1 = a1 / L;
            } else {
                f0 = 1.0f / l;
            }
            if (!ok) break;
            const int h = bh % H, row0 = (bh / H) * S;
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
                if (qpos < S) {                           // rows of a half last block beyond S are not stored
#pragma unroll
                    for (int g = 0; g < 2; ++g) reinterpret_cast<uint4*>(orow + c * 16)[g] = f_to_h8(o + 8 * g);
                }
            }
            if (wg == 0 && qpos < S) LSE[(size_t)bh * S + qpos] = (M + __log2f(L)) * 0.6931471805599453f;
            // O is out of TMEM: the next tile's first PV may overwrite it
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_free);
            jb += nkv;
        }
    }
    fence_before();
    __syncthreads();
    fence_after();
    if (threadIdx.x == 0 && *abort_flag) atomicExch(err, RBK_ERR_TIMEOUT);
    if (warp == 1) tmem_free(tmem, Cf::TMEM_COLS);
}

}  // namespace attn_tc

// Used by rbk_attn_fwd (attn.cu) for d_head 64 or 128 and S % 64 == 0.
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
        // all shared memory for the CTAS_PER_SM CTAs an SM hosts (the L1 split otherwise decides)
        RBK_CUDA(cudaFuncSetAttribute(flash_fwd_tc_kernel<HD>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                      (int)cudaSharedmemCarveoutMaxShared));
        set_dev = ctx->device;
    }
    // persistent: one CTA per resident slot (CTAS_PER_SM per SM, the launch bound), tiles from a
    // device counter that the last CTA re-arms; a CTA that cannot be resident only starts late
    const int BH = B * H, nqb = (S + BQ - 1) / BQ;
    const long ntiles = (long)nqb * BH;
    const long slots = (long)ctx->num_sms * FwdCfg<HD>::CTAS_PER_SM;
    const int grid = (int)(ntiles < slots ? ntiles : slots);
    int hpg = (2 * grid) / nqb;                       // heads per group: about two tiles per CTA
    if (hpg < 1) hpg = 1;
    if (hpg > BH) hpg = BH;
    RBK_CUDA(launch_pdl(flash_fwd_tc_kernel<HD>, dim3(grid), dim3(FwdCfg<HD>::THREADS), FwdCfg<HD>::SMEM, st, tmq,
                        tmkv, (half*)o, lse, S, H, BH, hpg, scale * 1.4426950408889634f,
                        ctx->tickets + kAttnFwdTile, ctx->tickets + kGemmError));
    RBK_LAUNCHED("flash_fwd_tc_kernel");
    return RBK_OK;
}

int attn_fwd_tc(rbk_ctx* ctx, void* o, float* lse, const void* qkv, int B, int S, int H, int dh, float scale,
                cudaStream_t st) {
    return dh == 64 ? attn_fwd_tc_hd<64>(ctx, o, lse, qkv, B, S, H, scale, st)
                    : attn_fwd_tc_hd<128>(ctx, o, lse, qkv, B, S, H, scale, st);
}

}  // namespace rbk
