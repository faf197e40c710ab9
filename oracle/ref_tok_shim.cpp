// ref_tok_shim.cpp — C entry points onto the reference's own GPU tokenizer
// kernels, compiled for the CPU from the reference sources where they lie
// (oracle/Makefile, target `ref`; the kernel section of
// src/tokenizer_cuda.cu is piped to g++ under ref_tok_shim.h).  Output goes to
// oracle/_ref/libreftok.so, which is git-ignored.
//
// TEST INFRASTRUCTURE ONLY: pins the tokenizer oracle (oracle/bpe.cpp) and
// generates tests/golden/bpe_ref.npz.
//
// Wrapped:
//   encode_kernel   src/tokenizer_cuda.cu:90-167, launched as encode_batch
//                   does (:287-332): one block of 256 threads per string,
//                   2 * 256 ints of shared memory
//   decode_kernel   src/tokenizer_cuda.cu:169-203, one thread per row
//                   (decode_batch, :334-348)
// The tables are laid out as the reference's builders do: the merge rules in
// merge order with priority = index (HostTokenizer::build_merge_trie,
// :408-454) and the inverse vocabulary as strings + offsets + lengths
// (build_inv_vocab_arrays, :488-505).
//
// Only the reference's defined domain is accepted: string lengths in
// [1, min(256, max_seq_len - 2)] for encode (a longer string reads shared
// memory no thread wrote, or writes past its row) and token ids inside the
// vocabulary for decode.  Outside it the calls return -1.
#include <chrono>
#include <vector>

#include "ref_tok_shim.h"

RefTokDim ref_tok_thread_idx, ref_tok_block_idx, ref_tok_block_dim;

namespace {
constexpr int kThreads = 256;  // encode_batch's launch (tokenizer_cuda.cu:320)
}  // namespace

int shared_tokens[2 * kThreads];  // the launch's dynamic shared memory (tokenizer_cuda.cu:321)

namespace {

GPUTokenizer make_tok(std::vector<MergeRule>& rules, const int* f, const int* s, const int* r, int n) {
    rules.resize(n);
    for (int i = 0; i < n; ++i) rules[i] = MergeRule{f[i], s[i], r[i], i};
    GPUTokenizer g;
    std::memset(&g, 0, sizeof(g));
    g.d_merge_rules = rules.data();
    g.num_merges = n;
    g.pad_id = 0;
    g.unk_id = 1;
    g.bos_id = 2;
    g.eos_id = 3;
    g.sep_id = 4;
    g.max_token_len = 32;
    return g;
}

void run_encode(const GPUTokenizer* g, const char* bytes, const int* offsets, const int* lengths, int batch, int* out,
                int* out_len, int max_seq_len) {
    ref_tok_block_dim = RefTokDim{kThreads, 1, 1};
    for (int b = 0; b < batch; ++b) {
        ref_tok_block_idx = RefTokDim{(unsigned)b, 0, 0};
        for (int t = kThreads - 1; t >= 0; --t) {  // thread 0 last: it reads every thread's write
            ref_tok_thread_idx = RefTokDim{(unsigned)t, 0, 0};
            encode_kernel(g, bytes, offsets, lengths, batch, out, out_len, max_seq_len);
        }
    }
}

}  // namespace

extern "C" {

int reftok_encode(const int* m_first, const int* m_second, const int* m_result, int n_merges, const char* bytes,
                  const int* offsets, const int* lengths, int batch, int* out, int* out_len, int max_seq_len) {
    for (int b = 0; b < batch; ++b)
        if (lengths[b] < 1 || lengths[b] > kThreads || lengths[b] > max_seq_len - 2) return -1;
    std::vector<MergeRule> rules;
    const GPUTokenizer g = make_tok(rules, m_first, m_second, m_result, n_merges);
    run_encode(&g, bytes, offsets, lengths, batch, out, out_len, max_seq_len);
    return 0;
}

// Seconds for `reps` encodes of the batch (the CPU cost of the reference's algorithm).
double reftok_time_encode(const int* m_first, const int* m_second, const int* m_result, int n_merges,
                          const char* bytes, const int* offsets, const int* lengths, int batch, int* out,
                          int* out_len, int max_seq_len, int reps) {
    for (int b = 0; b < batch; ++b)
        if (lengths[b] < 1 || lengths[b] > kThreads || lengths[b] > max_seq_len - 2) return -1.0;
    std::vector<MergeRule> rules;
    const GPUTokenizer g = make_tok(rules, m_first, m_second, m_result, n_merges);
    const auto t0 = std::chrono::steady_clock::now();
    for (int i = 0; i < reps; ++i) run_encode(&g, bytes, offsets, lengths, batch, out, out_len, max_seq_len);
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

// tokens: row b at tokens + b * lengths[b], as decode_kernel addresses them (tokenizer_cuda.cu:182).
int reftok_decode(const char* inv_bytes, const int* inv_offsets, const int* inv_lengths, int vocab_size,
                  const int* tokens, const int* lengths, int batch, char* out, int max_string_len) {
    for (int b = 0; b < batch; ++b) {
        const int* row = tokens + (long)b * lengths[b];
        for (int i = 0; i < lengths[b]; ++i) {
            if (row[i] == 3 || row[i] == 0) break;
            if (row[i] < 0 || row[i] >= vocab_size) return -1;
        }
    }
    std::vector<MergeRule> none;
    GPUTokenizer g = make_tok(none, nullptr, nullptr, nullptr, 0);
    g.vocab_size = vocab_size;
    g.d_inv_vocab_strings = const_cast<char*>(inv_bytes);
    g.d_inv_vocab_offsets = const_cast<int*>(inv_offsets);
    g.d_inv_vocab_lengths = const_cast<int*>(inv_lengths);
    ref_tok_block_dim = RefTokDim{1, 1, 1};
    ref_tok_thread_idx = RefTokDim{0, 0, 0};
    for (int b = 0; b < batch; ++b) {
        ref_tok_block_idx = RefTokDim{(unsigned)b, 0, 0};
        decode_kernel(&g, tokens, lengths, batch, out, max_string_len);
    }
    return 0;
}

}  // extern "C"
