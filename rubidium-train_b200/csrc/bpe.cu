// bpe.cu — the GPU BPE tokenizer: batch encode (bytes -> token rows) and batch decode
// (token rows -> strings), the data path of src/tokenizer_cuda.cu:90-203 rebuilt for sm_100a.
//
// Semantics (identical to the reference on its defined domain):
//   - byte c -> token c + 5, after the five special ids PAD 0, UNK 1, BOS 2, EOS 3, SEP 4
//     (vocab_lookup, tokenizer_cuda.cu:38-43);
//   - a pair (a, b) merges into the result of the FIRST rule in rule order with that pair
//     (find_merge, :75-84);
//   - merge passes run greedily left to right (merge a pair and step 2, else keep and step 1)
//     until a pass merges nothing, then EOS is appended (encode_kernel, :121-166);
//   - decode appends each token's string until EOS or PAD, skipping a token whose string would
//     not leave room for the NUL, then NUL-terminates (decode_kernel, :169-203).
// Where the reference is undefined (empty strings, strings of max_seq_len-1 bytes or more,
// the row past the EOS, decode row addressing, ids outside the vocabulary) the contract is
// stated at each entry point in rbk.h.
//
// Design.  The reference runs every pass serially on thread 0 of a block and scans the whole
// rule array for every pair (O(rules) per lookup).  Here:
//   - the rules live in an open-addressed hash table (load <= 1/4, linear probing) of 8-byte
//     slots {first | second << 16, result} for vocabularies of up to 65535 ids (the reference's
//     MAX_VOCAB_SIZE range; 2 MB for 50K rules) or 16-byte slots {first, second, result, 0}
//     above that: one L1/L2 load answers almost every lookup, and duplicate pairs keep the first
//     rule because the host inserts in rule order and skips pairs already present;
//   - one CTA of 256 threads owns a string (one warp, for rows of at most 257 tokens); each
//     pass is data-parallel: every thread looks up the pairs of its chunk of positions, and
//     the greedy left-to-right choice becomes a prefix computation.  Whether position p is consumed depends only on whether the pair
//     at p-1 merged, so a chunk is a map of that one-bit state (2 bits) together with how
//     many tokens it emits for either input state; composing these maps is associative, so
//     one block-wide scan of a packed 32-bit value gives every thread its input state and
//     its output offset, and the pass compacts in place in shared memory;
//   - the string stays in shared memory across passes; global memory sees the bytes once
//     and the finished row once (int4 stores, PAD-filled).
// Decode is one warp per row: a ballot finds the stop token, a warp scan of the string
// lengths gives every token its output position, and each lane copies its token's bytes.
// Only if a token would overflow the row does the rest of the row fall back to one lane
// (the reference's skip-and-continue rule is inherently sequential).
#include <condition_variable>
#include <functional>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "common.cuh"

// Host threads that pack the strings of large rbk_bpe_encode_batch calls, started on the first
// such call and kept until the handle is destroyed (spawning threads per call costs ~0.1-0.3 ms
// a round).  run(fn) calls fn(k) for k = 0 .. workers, the calling thread taking the last one.
struct rbk_bpe_pool {
    std::vector<std::thread> threads;
    std::mutex mu;
    std::condition_variable wake, idle;
    std::function<void(int)> job;
    unsigned gen = 0;
    int pending = 0;
    bool stop = false;

    // as many workers as the system grants, up to `workers` (none: the caller packs alone)
    explicit rbk_bpe_pool(int workers) {
        for (int k = 0; k < workers; ++k) {
            try {
                spawn(k);
            } catch (...) {
                break;
            }
        }
    }
    void spawn(int k) {
        threads.emplace_back([this, k] {
            unsigned seen = 0;
            for (;;) {
                std::function<void(int)> fn;
                {
                    std::unique_lock<std::mutex> lk(mu);
                    wake.wait(lk, [&] { return stop || gen != seen; });
                    if (stop) return;
                    seen = gen;
                    fn = job;
                }
                fn(k);
                std::lock_guard<std::mutex> lk(mu);
                if (--pending == 0) idle.notify_one();
            }
        });
    }
    int workers() const { return (int)threads.size(); }
    void run(const std::function<void(int)>& fn) {
        {
            std::lock_guard<std::mutex> lk(mu);
            job = fn;
            pending = workers();
            ++gen;
        }
        wake.notify_all();
        fn(workers());
        std::unique_lock<std::mutex> lk(mu);
        idle.wait(lk, [&] { return pending == 0; });
    }
    ~rbk_bpe_pool() {
        {
            std::lock_guard<std::mutex> lk(mu);
            stop = true;
        }
        wake.notify_all();
        for (auto& t : threads) t.join();
    }
};

struct rbk_bpe {
    int device = 0;
    int vocab_size = 0;
    int n_rules = 0;        // distinct usable pairs in the table
    uint32_t mask = 0;      // table slots - 1
    bool wide = false;      // 16-byte slots (vocabularies above 65535 ids), else 8-byte slots
    void* table = nullptr;  // device pair table (PairSlot<wide>)
    int2* inv = nullptr;    // device: {offset, length} of every id's string
    uint8_t* inv_bytes = nullptr;
    // host-string staging of rbk_bpe_encode_batch, double-buffered
    struct Slot {
        uint8_t* host = nullptr;  // pinned
        uint8_t* dev = nullptr;
        size_t cap = 0;
        cudaEvent_t done = nullptr;  // the slot's last copy and kernel have finished
        bool live = false;
    } slot[2];
    int next_slot = 0;
    std::unique_ptr<rbk_bpe_pool> pool;  // host packing threads (large batches)
};

namespace rbk {
namespace {

constexpr int kBpeThreads = 256;
constexpr int kPadId = 0;
constexpr int kEosId = 3;
constexpr int kByteBase = 5;
constexpr int kMaxItems = 32;  // positions per thread: strings of up to 256 * 32 tokens
constexpr int kDecodeWarps = 8;
constexpr int kWarpTokens = 256;  // longest string of the warp-per-string encode

// The pair hash: both ids multiplied by xxHash32's primes 1 and 2 (plus prime 5), then a
// xorshift-multiply avalanche; 32-bit arithmetic only (a few instructions per lookup).
__host__ __device__ __forceinline__ uint32_t pair_hash(int a, int b) {
    uint32_t h = ((uint32_t)a * 0x9E3779B1u) ^ ((uint32_t)b * 0x85EBCA77u + 0x165667B1u);
    h ^= h >> 15;
    h *= 0x2C1B3C6Du;
    h ^= h >> 13;
    return h;
}

// Pair-table slots.  Narrow (vocabularies of at most 65535 ids, the reference's
// MAX_VOCAB_SIZE range): 8 bytes {first | second << 16, result}, key 0xffffffff empty.  Wide:
// 16 bytes {first, second, result, 0}, first = -1 empty.
template <bool kWide>
struct PairSlot;
template <>
struct PairSlot<false> {
    using T = uint2;
    static __host__ __device__ T vacant() { return make_uint2(0xffffffffu, 0u); }
    static __host__ __device__ T make(int a, int b, int r) { return make_uint2((uint32_t)a | ((uint32_t)b << 16), (uint32_t)r); }
    static __host__ __device__ bool is_vacant(T e) { return e.x == 0xffffffffu; }
    static __host__ __device__ bool holds(T e, int a, int b) { return e.x == ((uint32_t)a | ((uint32_t)b << 16)); }
    static __host__ __device__ int result(T e) { return (int)e.y; }
};
template <>
struct PairSlot<true> {
    using T = int4;
    static __host__ __device__ T vacant() { return make_int4(-1, -1, -1, 0); }
    static __host__ __device__ T make(int a, int b, int r) { return make_int4(a, b, r, 0); }
    static __host__ __device__ bool is_vacant(T e) { return e.x < 0; }
    static __host__ __device__ bool holds(T e, int a, int b) { return e.x == a && e.y == b; }
    static __host__ __device__ int result(T e) { return e.z; }
};

// The rest of a probe sequence whose first slot (at index i) neither matched nor was vacant.
template <bool kWide>
__device__ __noinline__ int probe_rest(const typename PairSlot<kWide>::T* __restrict__ table, uint32_t mask, uint32_t i,
                                       int a, int b) {
    using S = PairSlot<kWide>;
    for (uint32_t n = 0; n < mask; ++n) {  // bounded by the table size; the table is never full
        i = (i + 1) & mask;
        const typename S::T e = __ldg(table + i);
        if (S::holds(e, a, b)) return S::result(e);
        if (S::is_vacant(e)) return -1;
    }
    return -1;
}

// ---- the chunk map of one pass --------------------------------------------------------
// bit 0: output state for input state 0, bit 1: for input state 1 (state = "the pair ending
// at the previous position merged"); bits 2-16: tokens emitted for input 0; bits 17-31: for
// input 1.  Counts stay below 2^15 (strings of at most 8192 tokens).
constexpr uint32_t kMapIdentity = 2u;

__device__ __forceinline__ uint32_t map_count(uint32_t m, uint32_t s) { return s ? (m >> 17) : ((m >> 2) & 0x7fffu); }

// `lo` covers earlier positions than `hi`
__device__ __forceinline__ uint32_t map_then(uint32_t lo, uint32_t hi) {
    const uint32_t o0 = lo & 1u, o1 = (lo >> 1) & 1u;
    const uint32_t c0 = map_count(lo, 0) + map_count(hi, o0);
    const uint32_t c1 = map_count(lo, 1) + map_count(hi, o1);
    return ((hi >> o0) & 1u) | (((hi >> o1) & 1u) << 1) | (c0 << 2) | (c1 << 17);
}

// One merge pass over the len tokens in s_tok, C positions per thread, on NT threads (the
// block, or one warp; NT C >= len); returns the new length (len when nothing merged).  Ends
// with a barrier of the NT threads: s_tok holds the new string.
template <int C, int NT, bool kWide>
__device__ __forceinline__ int merge_pass(int* s_tok, uint32_t* s_warp, int len,
                                          const typename PairSlot<kWide>::T* __restrict__ table, uint32_t mask) {
    using S = PairSlot<kWide>;
    static_assert(NT == 32 || NT == kBpeThreads, "a pass runs on one warp or on the whole block");
    const int tid = threadIdx.x % NT, lane = tid & 31, warp = tid >> 5;
    const int p0 = tid * C;
    int t[C], m[C];
    // the chunk, as 16- or 8-byte vectors (p0 is a multiple of C; every vector that starts below
    // len ends inside s_tok, whose size is a multiple of 4 ints)
    if constexpr (C >= 4) {
#pragma unroll
        for (int g = 0; g < C; g += 4) {
            int4 v = make_int4(-1, -1, -1, -1);
            if (p0 + g < len) v = *reinterpret_cast<const int4*>(s_tok + p0 + g);
            t[g] = v.x;
            t[g + 1] = v.y;
            t[g + 2] = v.z;
            t[g + 3] = v.w;
        }
    } else if constexpr (C == 2) {
        int2 v = make_int2(-1, -1);
        if (p0 < len) v = *reinterpret_cast<const int2*>(s_tok + p0);
        t[0] = v.x;
        t[1] = v.y;
    } else {
        t[0] = p0 < len ? s_tok[p0] : -1;
    }
#pragma unroll
    for (int k = 0; k < C; ++k)
        if (p0 + k >= len) t[k] = -1;
    // the token after the chunk is the next thread's first (a shuffle: s_tok read at stride C
    // would be a C-way bank conflict); the warp's last lane reads it
    int after = __shfl_down_sync(0xffffffffu, t[0], 1);
    if (lane == 31) after = (p0 + C < len) ? s_tok[p0 + C] : -1;
    // pair lookups: the first probes of up to 4 positions in flight together (more costs registers,
    // and so blocks per SM)
#pragma unroll
    for (int g = 0; g < C; g += (C < 4 ? C : 4)) {
        constexpr int G = C < 4 ? C : 4;
        typename S::T e[G];
        uint32_t idx[G];
#pragma unroll
        for (int j = 0; j < G; ++j) {
            const int k = g + j;
            const int second = (k + 1 < C) ? t[k + 1] : after;
            idx[j] = pair_hash(t[k], second) & mask;
            e[j] = (p0 + k + 1 < len) ? __ldg(table + idx[j]) : S::vacant();
        }
#pragma unroll
        for (int j = 0; j < G; ++j) {
            const int k = g + j;
            const int second = (k + 1 < C) ? t[k + 1] : after;
            int r = -1;
            if (p0 + k + 1 < len) {
                if (S::holds(e[j], t[k], second)) r = S::result(e[j]);
                else if (!S::is_vacant(e[j])) r = probe_rest<kWide>(table, mask, idx[j], t[k], second);
            }
            m[k] = r;
        }
    }
    // this chunk's map, by running it from both input states
    uint32_t f0 = 0, f1 = 1, n0 = 0, n1 = 0;
#pragma unroll
    for (int k = 0; k < C; ++k) {
        if (p0 + k < len) {
            const uint32_t has = m[k] >= 0;
            n0 += !f0;
            n1 += !f1;
            f0 = has & !f0;
            f1 = has & !f1;
        }
    }
    uint32_t v = f0 | (f1 << 1) | (n0 << 2) | (n1 << 17);
    // block-wide scan of the maps, left to right: warps, then the 8 warp maps
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const uint32_t o = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v = map_then(o, v);
    }
    uint32_t excl = __shfl_up_sync(0xffffffffu, v, 1);
    if (lane == 0) excl = kMapIdentity;
    uint32_t total;
    if constexpr (NT == 32) {
        total = __shfl_sync(0xffffffffu, v, 31);
        __syncwarp();
    } else {
        if (lane == 31) s_warp[warp] = v;
        __syncthreads();
        uint32_t x = lane < NT / 32 ? s_warp[lane] : kMapIdentity;
#pragma unroll
        for (int d = 1; d < NT / 32; d <<= 1) {
            const uint32_t o = __shfl_up_sync(0xffffffffu, x, d);
            if (lane >= d) x = map_then(o, x);
        }
        const uint32_t pre = __shfl_sync(0xffffffffu, x, warp > 0 ? warp - 1 : 0);  // used from warp 1 on
        total = __shfl_sync(0xffffffffu, x, NT / 32 - 1);
        if (warp > 0) excl = map_then(pre, excl);
    }
    // compact in place: every read of s_tok happened before the barrier above
    uint32_t st = excl & 1u;
    int o = (int)map_count(excl, 0);
#pragma unroll
    for (int k = 0; k < C; ++k) {
        if (p0 + k < len) {
            const uint32_t chosen = (m[k] >= 0) & !st;
            if (!st) s_tok[o++] = chosen ? m[k] : t[k];
            st = chosen;
        }
    }
    if constexpr (NT == 32) __syncwarp();
    else __syncthreads();
    return (int)map_count(total, 0);
}

// Strings of up to 256 K tokens (max_seq_len - 1 <= 256 K).  Each pass runs with the fewest
// positions per thread that cover the current length, so later, shorter passes cost less.
template <int K, bool kWide>
__global__ void __launch_bounds__(kBpeThreads, K <= 8 ? 6 : 1) bpe_encode_kernel(
    const typename PairSlot<kWide>::T* __restrict__ table, uint32_t mask, const uint8_t* __restrict__ bytes,
    const int64_t* __restrict__ offsets, const int* __restrict__ lengths, int* __restrict__ out,
    int* __restrict__ out_len, int max_seq_len, int* __restrict__ n_truncated) {
    __shared__ __align__(16) int s_tok[kBpeThreads * K];
    __shared__ uint32_t s_warp[kBpeThreads / 32];
    const int b = blockIdx.x;
    const int tid = threadIdx.x;

    int len = max(lengths[b], 0);
    if (len > max_seq_len - 1) {
        if (tid == 0 && n_truncated) atomicAdd(n_truncated, 1);
        len = max_seq_len - 1;
    }
    const uint8_t* src = bytes + offsets[b];
    for (int i = tid; i < len; i += kBpeThreads) s_tok[i] = (int)src[i] + kByteBase;
    __syncthreads();

    // Every pass that continues shortens the string, so at most len passes run.
    while (len > 1) {
        int nl;
        if (len <= kBpeThreads) nl = merge_pass<1, kBpeThreads, kWide>(s_tok, s_warp, len, table, mask);
        else if (K < 4 || len <= 2 * kBpeThreads) nl = merge_pass<(K < 2 ? 1 : 2), kBpeThreads, kWide>(s_tok, s_warp, len, table, mask);
        else if (K < 8 || len <= 4 * kBpeThreads) nl = merge_pass<(K < 4 ? 1 : 4), kBpeThreads, kWide>(s_tok, s_warp, len, table, mask);
        else if (K < 16 || len <= 8 * kBpeThreads) nl = merge_pass<(K < 8 ? 1 : 8), kBpeThreads, kWide>(s_tok, s_warp, len, table, mask);
        else if (K < 32 || len <= 16 * kBpeThreads)
            nl = merge_pass<(K < 16 ? 1 : 16), kBpeThreads, kWide>(s_tok, s_warp, len, table, mask);
        else nl = merge_pass<K, kBpeThreads, kWide>(s_tok, s_warp, len, table, mask);
        if (nl == len) break;
        len = nl;
    }

    // the finished row: tokens, EOS, PAD to max_seq_len
    int* row = out + (int64_t)b * max_seq_len;
    if ((max_seq_len & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
        int4* row4 = reinterpret_cast<int4*>(row);
        for (int q = tid; q < max_seq_len / 4; q += kBpeThreads) {
            int v4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int i = 4 * q + j;
                v4[j] = i < len ? s_tok[i] : (i == len ? kEosId : kPadId);
            }
            row4[q] = make_int4(v4[0], v4[1], v4[2], v4[3]);
        }
    } else {
        for (int i = tid; i < max_seq_len; i += kBpeThreads)
            row[i] = i < len ? s_tok[i] : (i == len ? kEosId : kPadId);
    }
    if (tid == 0) out_len[b] = len + 1;
}

// Strings of at most 256 tokens (max_seq_len <= 257, the reference kernel's one-block domain):
// one warp per string, 8 strings per block; passes synchronise the warp only.
template <bool kWide>
__global__ void __launch_bounds__(kBpeThreads, 5) bpe_encode_warp_kernel(
    const typename PairSlot<kWide>::T* __restrict__ table, uint32_t mask, const uint8_t* __restrict__ bytes,
    const int64_t* __restrict__ offsets, const int* __restrict__ lengths, int batch, int* __restrict__ out,
    int* __restrict__ out_len, int max_seq_len, int* __restrict__ n_truncated) {
    __shared__ __align__(16) int s_all[kBpeThreads / 32][kWarpTokens];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x * (kBpeThreads / 32) + warp;
    if (b >= batch) return;
    int* s_tok = s_all[warp];
    int len = max(lengths[b], 0);
    if (len > max_seq_len - 1) {
        if (lane == 0 && n_truncated) atomicAdd(n_truncated, 1);
        len = max_seq_len - 1;
    }
    const uint8_t* src = bytes + offsets[b];
    for (int i = lane; i < len; i += 32) s_tok[i] = (int)src[i] + kByteBase;
    __syncwarp();
    while (len > 1) {
        int nl;
        if (len <= 32) nl = merge_pass<1, 32, kWide>(s_tok, nullptr, len, table, mask);
        else if (len <= 64) nl = merge_pass<2, 32, kWide>(s_tok, nullptr, len, table, mask);
        else if (len <= 128) nl = merge_pass<4, 32, kWide>(s_tok, nullptr, len, table, mask);
        else nl = merge_pass<8, 32, kWide>(s_tok, nullptr, len, table, mask);
        if (nl == len) break;
        len = nl;
    }
    int* row = out + (int64_t)b * max_seq_len;
    if ((max_seq_len & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
        int4* row4 = reinterpret_cast<int4*>(row);
        for (int q = lane; q < max_seq_len / 4; q += 32) {
            int v4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int i = 4 * q + j;
                v4[j] = i < len ? s_tok[i] : (i == len ? kEosId : kPadId);
            }
            row4[q] = make_int4(v4[0], v4[1], v4[2], v4[3]);
        }
    } else {
        for (int i = lane; i < max_seq_len; i += 32) row[i] = i < len ? s_tok[i] : (i == len ? kEosId : kPadId);
    }
    if (lane == 0) out_len[b] = len + 1;
}

// One warp per row.  ld > 0: rows ld tokens apart, at most ld read; ld == 0: row r at
// r * lengths[r] (the reference's addressing).  The next 32 tokens are loaded while the current
// ones are placed, so the token -> string-table -> bytes chain is not the critical path.
__global__ void __launch_bounds__(32 * kDecodeWarps) bpe_decode_kernel(
    const int2* __restrict__ inv, const uint8_t* __restrict__ inv_bytes, int vocab, const int* __restrict__ tokens,
    int64_t ld, const int* __restrict__ lengths, int batch, char* __restrict__ out, int max_string_len,
    int* __restrict__ n_bad) {
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * kDecodeWarps + (threadIdx.x >> 5);
    if (r >= batch) return;
    const int len_r = lengths[r];
    int n = max(len_r, 0);
    if (ld > 0 && n > ld) n = (int)ld;
    const int* tr = tokens + (ld > 0 ? (int64_t)r * ld : (int64_t)r * len_r);
    char* const o = out + (int64_t)r * max_string_len;
    int w = 0, bad = 0;
    int tail = -1;  // first token of the serial tail, if a token did not fit
    int t_next = lane < n ? __ldg(tr + lane) : kPadId;
    for (int base = 0; base < n; base += 32) {
        const int i = base + lane;
        const int t = t_next;
        t_next = i + 32 < n ? __ldg(tr + i + 32) : kPadId;
        const unsigned stop = __ballot_sync(0xffffffffu, i >= n || t == kEosId || t == kPadId);
        const int first_stop = stop ? __ffs(stop) - 1 : 32;
        const bool act = lane < first_stop;
        const bool ok = act && t >= 0 && t < vocab;
        const int2 e = ok ? __ldg(inv + t) : make_int2(0, 0);
        int incl = e.y;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int x = __shfl_up_sync(0xffffffffu, incl, d);
            if (lane >= d) incl += x;
        }
        const unsigned fail = __ballot_sync(0xffffffffu, act && w + incl >= max_string_len);
        const int first_fail = fail ? __ffs(fail) - 1 : 32;
        // ids outside the vocabulary before the stop; from a failing token on, the serial tail counts
        bad += __popc(__ballot_sync(0xffffffffu, act && !ok && lane < first_fail));
        if (act && lane < first_fail) {
            const uint8_t* s = inv_bytes + e.x;
            char* d = o + w + incl - e.y;
            for (int j = 0; j < e.y; ++j) d[j] = (char)__ldg(s + j);
        }
        if (first_fail < 32) {
            w += __shfl_sync(0xffffffffu, incl - e.y, first_fail);
            tail = base + first_fail + 1;
            break;
        }
        w += __shfl_sync(0xffffffffu, incl, first_stop == 32 ? 31 : max(first_stop - 1, 0)) * (first_stop > 0);
        if (first_stop < 32) break;
    }
    if (lane == 0) {
        if (tail >= 0) {  // the rest in order: each token that still fits is appended
            for (int i = tail; i < n; ++i) {
                const int t = tr[i];
                if (t == kEosId || t == kPadId) break;
                if (t < 0 || t >= vocab) {
                    ++bad;
                    continue;
                }
                const int2 e = inv[t];
                if (w + e.y < max_string_len) {
                    for (int j = 0; j < e.y; ++j) o[w + j] = (char)inv_bytes[e.x + j];
                    w += e.y;
                }
            }
        }
        o[w] = '\0';
        if (bad && n_bad) atomicAdd(n_bad, bad);
    }
}

// smallest items-per-thread instance that holds max_seq_len - 1 tokens
int encode_items(int max_seq_len) {
    int k = 1;
    while (kBpeThreads * k < max_seq_len - 1) k *= 2;
    return k;
}

template <bool kWide>
int launch_encode_as(const rbk_bpe* t, const uint8_t* bytes, const int64_t* offsets, const int* lengths, int batch,
                     int* out, int* out_len, int max_seq_len, int* n_truncated, cudaStream_t st) {
    using T = typename PairSlot<kWide>::T;
    const T* table = static_cast<const T*>(t->table);
    if (max_seq_len - 1 <= kWarpTokens) {
        const int per = kBpeThreads / 32;
        bpe_encode_warp_kernel<kWide><<<(batch + per - 1) / per, kBpeThreads, 0, st>>>(
            table, t->mask, bytes, offsets, lengths, batch, out, out_len, max_seq_len, n_truncated);
        RBK_LAUNCHED("bpe_encode_warp_kernel");
        return RBK_OK;
    }
    const dim3 grid(batch), block(kBpeThreads);
    switch (encode_items(max_seq_len)) {
#define RBK_BPE_CASE(K)                                                                                          \
    case K:                                                                                                      \
        bpe_encode_kernel<K, kWide><<<grid, block, 0, st>>>(table, t->mask, bytes, offsets, lengths, out, out_len, \
                                                           max_seq_len, n_truncated);                            \
        break;
        RBK_BPE_CASE(2)
        RBK_BPE_CASE(4)
        RBK_BPE_CASE(8)
        RBK_BPE_CASE(16)
        RBK_BPE_CASE(32)
#undef RBK_BPE_CASE
        default:
            set_error("rbk_bpe: max_seq_len %d above %d", max_seq_len, kBpeThreads * kMaxItems + 1);
            return RBK_ERR_INVALID;
    }
    RBK_LAUNCHED("bpe_encode_kernel");
    return RBK_OK;
}

int launch_encode(const rbk_bpe* t, const uint8_t* bytes, const int64_t* offsets, const int* lengths, int batch,
                  int* out, int* out_len, int max_seq_len, int* n_truncated, cudaStream_t st) {
    return t->wide ? launch_encode_as<true>(t, bytes, offsets, lengths, batch, out, out_len, max_seq_len, n_truncated, st)
                   : launch_encode_as<false>(t, bytes, offsets, lengths, batch, out, out_len, max_seq_len, n_truncated,
                                             st);
}

// Insert the rules in rule order (a pair already present keeps its earlier rule; a rule whose
// pair holds an id no token can carry never fires and is dropped) and upload the table.
template <bool kWide>
int build_table(rbk_bpe* t, const int* f, const int* s2, const int* r, int n, uint32_t slots) {
    using S = PairSlot<kWide>;
    std::vector<typename S::T> table(slots, S::vacant());
    const uint32_t mask = slots - 1;
    int n_rules = 0;
    for (int i = 0; i < n; ++i) {
        const int a = f[i], b = s2[i];
        if (a < 0 || b < 0 || a >= t->vocab_size || b >= t->vocab_size) continue;
        uint32_t j = pair_hash(a, b) & mask;
        while (!S::is_vacant(table[j]) && !S::holds(table[j], a, b)) j = (j + 1) & mask;
        if (!S::is_vacant(table[j])) continue;
        table[j] = S::make(a, b, r[i]);
        ++n_rules;
    }
    t->n_rules = n_rules;
    t->mask = mask;
    t->wide = kWide;
    if (cudaMalloc(&t->table, sizeof(typename S::T) * slots) != cudaSuccess) {
        cudaGetLastError();
        t->table = nullptr;
        set_error("rbk_bpe_create: device allocation of the pair table failed");
        return RBK_ERR_NOMEM;
    }
    RBK_CUDA(cudaMemcpy(t->table, table.data(), sizeof(typename S::T) * slots, cudaMemcpyHostToDevice));
    return RBK_OK;
}

int check_device(const rbk_bpe* t) {
    int cur = -1;
    RBK_CUDA(cudaGetDevice(&cur));
    RBK_REQUIRE(cur == t->device, "rbk_bpe: the current device is %d, the tokenizer lives on device %d", cur,
                t->device);
    return RBK_OK;
}

void free_slot(rbk_bpe::Slot& s) {
    if (s.done) {
        if (s.live) cudaEventSynchronize(s.done);
        cudaEventDestroy(s.done);
    }
    if (s.host) cudaFreeHost(s.host);
    if (s.dev) cudaFree(s.dev);
    s = rbk_bpe::Slot{};
}

void free_bpe(rbk_bpe* t) {
    t->pool.reset();
    for (auto& s : t->slot) free_slot(s);
    if (t->table) cudaFree(t->table);
    if (t->inv) cudaFree(t->inv);
    if (t->inv_bytes) cudaFree(t->inv_bytes);
    delete t;
}

}  // namespace
}  // namespace rbk

using namespace rbk;

extern "C" {

int rbk_bpe_create(rbk_bpe** out, int device, int vocab_size, const char* inv_bytes, int64_t inv_bytes_size,
                   const int* inv_offsets, const int* inv_lengths, const int* merge_first, const int* merge_second,
                   const int* merge_result, int num_merges) {
    RBK_REQUIRE(out, "rbk_bpe_create: null handle pointer");
    *out = nullptr;
    RBK_REQUIRE(vocab_size >= 256 + kByteBase, "rbk_bpe_create: vocab_size %d below the 261 ids of specials + bytes",
                vocab_size);
    RBK_REQUIRE(inv_offsets && inv_lengths && (inv_bytes || inv_bytes_size == 0) && inv_bytes_size >= 0 &&
                    inv_bytes_size < (int64_t)1 << 31,
                "rbk_bpe_create: bad inverse vocabulary (null table or over 2 GiB of strings)");
    RBK_REQUIRE(num_merges >= 0 && (num_merges == 0 || (merge_first && merge_second && merge_result)),
                "rbk_bpe_create: bad merge rules");
    std::vector<int2> inv(vocab_size);
    for (int i = 0; i < vocab_size; ++i) {
        RBK_REQUIRE(inv_lengths[i] >= 0 && inv_offsets[i] >= 0 && (int64_t)inv_offsets[i] + inv_lengths[i] <=
                                                                       inv_bytes_size,
                    "rbk_bpe_create: string of id %d (offset %d, length %d) outside the %lld string bytes", i,
                    inv_offsets[i], inv_lengths[i], (long long)inv_bytes_size);
        inv[i] = make_int2(inv_offsets[i], inv_lengths[i]);
    }
    for (int i = 0; i < num_merges; ++i)
        RBK_REQUIRE(merge_result[i] >= 0 && merge_result[i] < vocab_size,
                    "rbk_bpe_create: rule %d yields id %d outside the vocabulary of %d", i, merge_result[i],
                    vocab_size);
    cudaDeviceProp prop;
    RBK_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10 || prop.minor != 0) {
        set_error("librbk is built for sm_100a (B200); device %d is sm_%d%d", device, prop.major, prop.minor);
        return RBK_ERR_UNSUPPORTED;
    }
    RBK_CUDA(cudaSetDevice(device));
    rbk_bpe* t = new rbk_bpe;
    t->device = device;
    t->vocab_size = vocab_size;
    // the pair table: load <= 1/4
    uint32_t slots = 1024;
    while (slots < 4ull * (uint64_t)num_merges) slots *= 2;
    const int rc = vocab_size <= 65535
                       ? build_table<false>(t, merge_first, merge_second, merge_result, num_merges, slots)
                       : build_table<true>(t, merge_first, merge_second, merge_result, num_merges, slots);
    if (rc != RBK_OK) {
        free_bpe(t);
        return rc;
    }
    const size_t nb = (size_t)std::max<int64_t>(inv_bytes_size, 1);
    if (cudaMalloc(&t->inv, sizeof(int2) * vocab_size) != cudaSuccess || cudaMalloc(&t->inv_bytes, nb) != cudaSuccess) {
        cudaGetLastError();
        free_bpe(t);
        set_error("rbk_bpe_create: device allocation of the tables failed");
        return RBK_ERR_NOMEM;
    }
    cudaError_t e = cudaMemcpy(t->inv, inv.data(), sizeof(int2) * vocab_size, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && inv_bytes_size > 0)
        e = cudaMemcpy(t->inv_bytes, inv_bytes, (size_t)inv_bytes_size, cudaMemcpyHostToDevice);
    for (auto& s : t->slot)
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming);
    if (e != cudaSuccess) {
        free_bpe(t);
        return cuda_fail(e, "rbk_bpe_create upload", __FILE__, __LINE__);
    }
    *out = t;
    return RBK_OK;
}

int rbk_bpe_destroy(rbk_bpe* t) {
    if (!t) return RBK_OK;
    int cur = -1;
    cudaGetDevice(&cur);
    cudaSetDevice(t->device);
    free_bpe(t);
    if (cur >= 0) cudaSetDevice(cur);
    return RBK_OK;
}

int rbk_bpe_num_rules(const rbk_bpe* t) { return t ? t->n_rules : 0; }

int rbk_bpe_encode(rbk_bpe* t, const uint8_t* bytes, const int64_t* offsets, const int* lengths, int batch,
                   int* out_tokens, int* out_lengths, int max_seq_len, int* n_truncated, void* stream) {
    RBK_REQUIRE(t, "rbk_bpe_encode: null tokenizer");
    RBK_REQUIRE(batch >= 0, "rbk_bpe_encode: negative batch");
    RBK_REQUIRE(max_seq_len >= 2 && max_seq_len <= kBpeThreads * kMaxItems + 1,
                "rbk_bpe_encode: max_seq_len %d outside [2, %d]", max_seq_len, kBpeThreads * kMaxItems + 1);
    if (batch == 0) return RBK_OK;
    RBK_REQUIRE(bytes && offsets && lengths && out_tokens && out_lengths, "rbk_bpe_encode: null pointer");
    RBK_TRY(check_device(t));
    return launch_encode(t, bytes, offsets, lengths, batch, out_tokens, out_lengths, max_seq_len, n_truncated,
                         as_stream(stream));
}

int rbk_bpe_encode_batch(rbk_bpe* t, const char* const* strings, int batch, int* out_tokens, int* out_lengths,
                         int max_seq_len, void* stream) {
    RBK_REQUIRE(t, "rbk_bpe_encode_batch: null tokenizer");
    RBK_REQUIRE(batch >= 0 && (batch == 0 || strings), "rbk_bpe_encode_batch: bad batch");
    RBK_REQUIRE(max_seq_len >= 2 && max_seq_len <= kBpeThreads * kMaxItems + 1,
                "rbk_bpe_encode_batch: max_seq_len %d outside [2, %d]", max_seq_len, kBpeThreads * kMaxItems + 1);
    if (batch == 0) return RBK_OK;
    RBK_REQUIRE(out_tokens && out_lengths, "rbk_bpe_encode_batch: null output");
    RBK_TRY(check_device(t));
    // staging layout: offsets (int64) | lengths (int32, padded to 8 bytes) | bytes
    for (int b = 0; b < batch; ++b) RBK_REQUIRE(strings[b], "rbk_bpe_encode_batch: string %d is null", b);
    // String lengths, then (below) the copy into pinned memory: both in slices on the handle's
    // host threads for large batches (one core scans or copies ~10 GB/s, below what the copy engine
    // takes).  A length above the row is kept as -1 and rejected before anything is staged.
    int nthr = 1;
    if (batch >= 1024) {
        if (!t->pool) {
            const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
            t->pool.reset(new rbk_bpe_pool((int)std::min<unsigned>(8u, hw) - 1));
        }
        nthr = t->pool->workers() + 1;
    }
    // fn(b0, b1) over nthr slices of [0, n), on the pool when there is more than one
    auto slices = [&](int n, const std::function<void(int, int)>& fn) {
        if (nthr == 1 || n < 1024) {
            fn(0, n);
            return;
        }
        t->pool->run([&](int k) { fn((int)((int64_t)n * k / nthr), (int)((int64_t)n * (k + 1) / nthr)); });
    };
    auto in_slices = [&](const std::function<void(int, int)>& fn) { slices(batch, fn); };
    std::vector<int> len(batch);
    in_slices([&](int b0, int b1) {
        for (int b = b0; b < b1; ++b) {
            const size_t l = strlen(strings[b]);
            len[b] = l <= (size_t)max_seq_len - 1 ? (int)l : -1;
        }
    });
    size_t total = 0;
    for (int b = 0; b < batch; ++b) {
        RBK_REQUIRE(len[b] >= 0, "rbk_bpe_encode_batch: string %d has %zu bytes, above max_seq_len - 1 = %d", b,
                    strlen(strings[b]), max_seq_len - 1);
        total += len[b];
    }
    const size_t off_bytes = sizeof(int64_t) * batch, len_bytes = (sizeof(int) * batch + 7) / 8 * 8;
    const size_t need = off_bytes + len_bytes + std::max<size_t>(total, 1);
    rbk_bpe::Slot& s = t->slot[t->next_slot];
    t->next_slot ^= 1;
    if (s.live) RBK_CUDA(cudaEventSynchronize(s.done));  // its previous copy and kernel are done
    s.live = false;
    if (s.cap < need) {
        if (s.host) RBK_CUDA(cudaFreeHost(s.host));
        if (s.dev) RBK_CUDA(cudaFree(s.dev));
        s.host = nullptr;
        s.dev = nullptr;
        s.cap = 0;
        const size_t cap = std::max<size_t>(need + need / 2, 1 << 16);
        if (cudaHostAlloc(&s.host, cap, cudaHostAllocDefault) != cudaSuccess || cudaMalloc(&s.dev, cap) != cudaSuccess) {
            cudaGetLastError();
            if (s.host) cudaFreeHost(s.host);
            s.host = nullptr;
            set_error("rbk_bpe_encode_batch: staging allocation of %zu bytes failed", cap);
            return RBK_ERR_NOMEM;
        }
        s.cap = cap;
    }
    int64_t* h_off = reinterpret_cast<int64_t*>(s.host);
    int* h_len = reinterpret_cast<int*>(s.host + off_bytes);
    uint8_t* h_bytes = s.host + off_bytes + len_bytes;
    size_t pos = 0;
    for (int b = 0; b < batch; ++b) {
        h_off[b] = (int64_t)pos;
        h_len[b] = len[b];
        pos += len[b];
    }
    // Offsets and lengths first; then the text in up to four parts: part p + 1 is packed on the
    // host while part p is copied and encoded (strings are independent: each part is one launch).
    cudaStream_t st = as_stream(stream);
    RBK_CUDA(cudaMemcpyAsync(s.dev, s.host, off_bytes + len_bytes, cudaMemcpyHostToDevice, st));
    const int parts = (batch >= 4096 && total >= ((size_t)8 << 20)) ? 4 : 1;
    const int64_t* d_off = reinterpret_cast<const int64_t*>(s.dev);
    const int* d_len = reinterpret_cast<const int*>(s.dev + off_bytes);
    int rc = RBK_OK;
    for (int p = 0; p < parts && rc == RBK_OK; ++p) {
        const int b0 = (int)((int64_t)batch * p / parts), b1 = (int)((int64_t)batch * (p + 1) / parts);
        if (b1 == b0) continue;
        const int n = b1 - b0;
        slices(n, [&](int c0, int c1) {
            for (int b = b0 + c0; b < b0 + c1; ++b) memcpy(h_bytes + h_off[b], strings[b], len[b]);
        });
        const size_t lo = (size_t)h_off[b0], hi = (size_t)h_off[b1 - 1] + len[b1 - 1];
        if (hi > lo)
            RBK_CUDA(cudaMemcpyAsync(s.dev + off_bytes + len_bytes + lo, h_bytes + lo, hi - lo, cudaMemcpyHostToDevice,
                                     st));
        rc = launch_encode(t, s.dev + off_bytes + len_bytes, d_off + b0, d_len + b0, n,
                           out_tokens + (int64_t)b0 * max_seq_len, out_lengths + b0, max_seq_len, nullptr, st);
    }
    RBK_CUDA(cudaEventRecord(s.done, st));
    s.live = true;
    return rc;
}

int rbk_bpe_decode_batch(rbk_bpe* t, const int* tokens, int64_t ld, const int* lengths, int batch, char* out,
                         int max_string_len, int* n_bad, void* stream) {
    RBK_REQUIRE(t, "rbk_bpe_decode_batch: null tokenizer");
    RBK_REQUIRE(batch >= 0 && ld >= 0 && max_string_len >= 1, "rbk_bpe_decode_batch: bad batch, ld or max_string_len");
    if (batch == 0) return RBK_OK;
    RBK_REQUIRE(tokens && lengths && out, "rbk_bpe_decode_batch: null pointer");
    RBK_TRY(check_device(t));
    const int blocks = (batch + kDecodeWarps - 1) / kDecodeWarps;
    bpe_decode_kernel<<<blocks, 32 * kDecodeWarps, 0, as_stream(stream)>>>(t->inv, t->inv_bytes, t->vocab_size,
                                                                          tokens, ld, lengths, batch, out,
                                                                          max_string_len, n_bad);
    RBK_LAUNCHED("bpe_decode_kernel");
    return RBK_OK;
}

}  // extern "C"
