// bpe.cpp — CPU restatement of the reference's GPU BPE tokenizer (encode and
// decode), linked into liboracle.so.
//
// TEST INFRASTRUCTURE ONLY: the checker the CUDA tokenizer is compared
// against; only tests/, __graft_entry__.smoke() and bench.py's CPU baseline
// leg load it.  Pinned against the reference's own kernels compiled for the
// CPU (oracle/ref_tok_shim.cpp -> _ref/libreftok.so) and the fixtures they
// generated (tests/golden/bpe_ref.npz).
//
// Restated (reference paths relative to its project):
//   byte -> token id   byte + 5, after the five special ids
//                      (vocab_lookup, src/tokenizer_cuda.cu:38-43)
//   pair lookup        the result of the FIRST rule, in rule order, whose
//                      (first_id, second_id) equals the pair, else none
//                      (find_merge, src/tokenizer_cuda.cu:75-84)
//   merge passes       greedy left-to-right passes: at each position, merge
//                      the pair and step 2, else keep the token and step 1;
//                      repeat while a pass merged something; then EOS (id 3)
//                      is appended and the length is tokens + 1
//                      (encode_kernel, src/tokenizer_cuda.cu:121-166)
//   decode             per row, append each token's string until EOS (3) or
//                      PAD (0); a token whose string would not leave room for
//                      the terminating NUL is skipped and the scan goes on;
//                      NUL-terminate (decode_kernel, src/tokenizer_cuda.cu:169-203)
//
// The contract on the cases the reference leaves undefined (shared with the
// CUDA path):
//   - an empty string encodes to [EOS], length 1 (the reference writes nothing);
//   - a string of max_seq_len-1 bytes is merged like any other (the reference's
//     pass guard, :128, skips the passes and leaves the row unwritten);
//   - a longer string is cut to its first max_seq_len-1 bytes and counted in
//     *n_truncated (the reference writes past the row);
//   - the row after the EOS is filled with PAD (the reference leaves the
//     intermediate pass results there);
//   - decode rows sit ld tokens apart; ld == 0 keeps the reference's
//     addressing, row b at b * lengths[b] (:182);
//   - a token id outside [0, vocab_size) adds no bytes and is counted in
//     *n_bad (the reference reads outside its tables).
#include <cstdint>
#include <cstring>
#include <unordered_map>
#include <vector>

namespace {

constexpr int kPad = 0;
constexpr int kEos = 3;
constexpr int kByteBase = 5;

uint64_t pair_key(int a, int b) { return ((uint64_t)(uint32_t)a << 32) | (uint32_t)b; }

struct Rules {
    std::unordered_map<uint64_t, int> first_result;
    Rules(const int* f, const int* s, const int* r, int n) {
        first_result.reserve((size_t)n * 2);
        for (int i = 0; i < n; ++i) first_result.emplace(pair_key(f[i], s[i]), r[i]);  // emplace keeps the first
    }
    int find(int a, int b) const {
        auto it = first_result.find(pair_key(a, b));
        return it == first_result.end() ? -1 : it->second;
    }
};

// one string: bytes -> tokens merged to the fixpoint (tokenizer_cuda.cu:115-160)
void encode_one(const Rules& rules, const unsigned char* s, int len, std::vector<int>& tok, std::vector<int>& nxt) {
    tok.resize(len);
    for (int i = 0; i < len; ++i) tok[i] = (int)s[i] + kByteBase;
    for (;;) {
        nxt.clear();
        bool merged = false;
        int r = 0;
        const int n = (int)tok.size();
        while (r < n - 1) {
            const int m = rules.find(tok[r], tok[r + 1]);
            if (m != -1) {
                nxt.push_back(m);
                r += 2;
                merged = true;
            } else {
                nxt.push_back(tok[r]);
                r += 1;
            }
        }
        if (r < n) nxt.push_back(tok[r]);
        tok.swap(nxt);
        if (!merged) break;
    }
}

}  // namespace

extern "C" {

// Encode `batch` byte strings (string b = bytes[offsets[b] .. offsets[b] + lengths[b])) into rows of
// max_seq_len token ids at out + b * max_seq_len; out_len[b] = tokens + 1 (the EOS).
int ora_bpe_encode(const int* m_first, const int* m_second, const int* m_result, int n_merges,
                   const unsigned char* bytes, const int64_t* offsets, const int* lengths, int batch, int* out,
                   int* out_len, int max_seq_len, int* n_truncated) {
    if (max_seq_len < 2 || batch < 0 || n_merges < 0) return -1;
    for (int b = 0; b < batch; ++b)
        if (lengths[b] < 0) return -1;
    const Rules rules(m_first, m_second, m_result, n_merges);
    int cut = 0;
    // strings are independent: one per OpenMP iteration (the thread count follows OMP_NUM_THREADS
    // or ora_set_threads)
#pragma omp parallel reduction(+ : cut)
    {
        std::vector<int> tok, nxt;
#pragma omp for schedule(dynamic, 16)
        for (int b = 0; b < batch; ++b) {
            int len = lengths[b];
            if (len > max_seq_len - 1) {
                len = max_seq_len - 1;
                ++cut;
            }
            encode_one(rules, bytes + offsets[b], len, tok, nxt);
            int* row = out + (size_t)b * max_seq_len;
            const int n = (int)tok.size();
            std::memcpy(row, tok.data(), sizeof(int) * n);
            row[n] = kEos;
            for (int i = n + 1; i < max_seq_len; ++i) row[i] = kPad;
            out_len[b] = n + 1;
        }
    }
    if (n_truncated) *n_truncated = cut;
    return 0;
}

// Decode `batch` token rows into NUL-terminated strings of at most max_string_len bytes at
// out + b * max_string_len (bytes after the NUL are left as they were).
int ora_bpe_decode(const unsigned char* inv_bytes, const int64_t* inv_offsets, const int* inv_lengths, int vocab_size,
                   const int* tokens, int64_t ld, const int* lengths, int batch, char* out, int max_string_len,
                   int* n_bad) {
    if (max_string_len < 1 || batch < 0 || ld < 0) return -1;
    int bad = 0;
    for (int b = 0; b < batch; ++b) {
        int n = lengths[b];
        if (n < 0) n = 0;
        if (ld > 0 && n > ld) n = (int)ld;
        const int* row = tokens + (ld > 0 ? (int64_t)b * ld : (int64_t)b * lengths[b]);
        char* o = out + (size_t)b * max_string_len;
        int w = 0;
        for (int i = 0; i < n; ++i) {
            const int t = row[i];
            if (t == kEos || t == kPad) break;
            if (t < 0 || t >= vocab_size) {
                ++bad;
                continue;
            }
            const int l = inv_lengths[t];
            if (w + l < max_string_len) {
                std::memcpy(o + w, inv_bytes + inv_offsets[t], l);
                w += l;
            }
        }
        o[w] = '\0';
    }
    if (n_bad) *n_bad = bad;
    return 0;
}

}  // extern "C"
