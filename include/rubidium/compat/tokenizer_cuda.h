// compat/tokenizer_cuda.h — the reference's "tokenizer_cuda.h" name (src/fine_tune.cu
// includes it): HostTokenizer, GPUTokenizer and the free functions of
// src/tokenizer_cuda.h:120-169, header-only over librbk's rbk_bpe_* calls.
//
// Same ids and rules as the reference (PAD 0, UNK 1, BOS 2, EOS 3, SEP 4; byte c -> c + 5;
// the first rule of a pair wins; greedy passes to a fixpoint; EOS appended; decode stops at
// EOS / PAD and skips a string that would not leave room for the NUL).  Differences, all
// where the reference is undefined or does not compile:
//   - the special ids and size limits are constants, not macros: the reference's PAD_ID ..
//     SEP_ID macros (tokenizer_cuda.h:20-24) expand inside HostTokenizer's members of the
//     same names (:102-106), so the reference header does not compile;
//   - HostTokenizer::load_from_json returns false, as the reference's does (:402-406): fill
//     vocab / inv_vocab / merges / vocab_size directly;
//   - encode_batch rejects a string of more than max_seq_len - 1 bytes (cudaErrorInvalidValue)
//     instead of writing past the row; encode_string cuts such a text to that many bytes;
//   - a row holds PAD after its EOS; an empty string encodes to [EOS];
//   - tokenizer_validate_roundtrip, declared but never defined by the reference (:169), is
//     defined here.
// Error codes: rbk statuses map to cudaError_t values; rbk_last_error() has the message.
// A GPUTokenizer* is, as in the reference, a small device allocation: the caller frees it
// with cudaFree after tokenizer_free_gpu.  Not thread-safe (one registry per process).
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "rbk.h"

constexpr int MAX_VOCAB_SIZE = 65536;
constexpr int MAX_MERGES = 60000;
constexpr int MAX_BATCH_SIZE = 256;
constexpr int MAX_SEQ_LEN = 2048;
constexpr int MAX_TOKEN_LEN = 32;
constexpr int PAD_ID = 0;
constexpr int UNK_ID = 1;
constexpr int BOS_ID = 2;
constexpr int EOS_ID = 3;
constexpr int SEP_ID = 4;

// The host-side tables (tokenizer_cuda.h:97-116).
struct HostTokenizer {
    std::unordered_map<std::string, int> vocab;
    std::unordered_map<int, std::string> inv_vocab;
    std::vector<std::pair<std::pair<int, int>, std::string>> merges;  // ((first, second), merged string)
    std::unordered_map<std::string, double> unigram_probs;
    int vocab_size = 0;

    const int PAD_ID = 0;
    const int UNK_ID = 1;
    const int BOS_ID = 2;
    const int EOS_ID = 3;
    const int SEP_ID = 4;

    bool load_from_json(const std::string&) { return false; }
};

// Opaque: the address of a device allocation that names the tokenizer's librbk handle.
struct GPUTokenizer {
    int unused;
};

namespace rubidium_tok_detail {

inline std::map<const GPUTokenizer*, rbk_bpe*>& registry() {
    static std::map<const GPUTokenizer*, rbk_bpe*> r;
    return r;
}

inline rbk_bpe* handle(const GPUTokenizer* t) {
    auto it = registry().find(t);
    return it == registry().end() ? nullptr : it->second;
}

inline cudaError_t to_cuda(int st) {
    switch (st) {
        case RBK_OK: return cudaSuccess;
        case RBK_ERR_INVALID: return cudaErrorInvalidValue;
        case RBK_ERR_NOMEM: return cudaErrorMemoryAllocation;
        case RBK_ERR_UNSUPPORTED: return cudaErrorNotSupported;
        default: return cudaErrorUnknown;
    }
}

}  // namespace rubidium_tok_detail

// tokenizer_init_gpu (tokenizer_cuda.cu:205-272): the tables of h_tok, laid out as the
// reference's build_inv_vocab_arrays / build_merge_trie lay them out (a merge's result is
// vocab[merged string], 0 when absent; ids without a string decode to nothing), on the
// current device.  The device id space covers the specials and bytes even for an empty table.
inline cudaError_t tokenizer_init_gpu(GPUTokenizer* d_tok, const HostTokenizer& h_tok) {
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return e;
    std::vector<int> first, second, result;
    first.reserve(h_tok.merges.size());
    int top = std::max(h_tok.vocab_size, 256 + 5);
    for (const auto& m : h_tok.merges) {
        auto it = h_tok.vocab.find(m.second);
        first.push_back(m.first.first);
        second.push_back(m.first.second);
        result.push_back(it == h_tok.vocab.end() ? 0 : it->second);
        top = std::max(top, result.back() + 1);
    }
    for (const auto& kv : h_tok.inv_vocab) top = std::max(top, kv.first + 1);
    std::vector<int> off(top, 0), len(top, 0);
    std::string bytes;
    for (int i = 0; i < top; ++i) {
        auto it = h_tok.inv_vocab.find(i);
        if (it == h_tok.inv_vocab.end()) continue;
        off[i] = (int)bytes.size();
        len[i] = (int)it->second.size();
        bytes += it->second;
    }
    rbk_bpe* t = nullptr;
    const int st = rbk_bpe_create(&t, device, top, bytes.data(), (int64_t)bytes.size(), off.data(), len.data(),
                                  first.data(), second.data(), result.data(), (int)first.size());
    if (st != RBK_OK) return rubidium_tok_detail::to_cuda(st);
    rubidium_tok_detail::registry()[d_tok] = t;
    return cudaSuccess;
}

// tokenizer_copy_to_device (tokenizer_cuda.cu:391-394).
inline cudaError_t tokenizer_copy_to_device(const HostTokenizer& h_tok, GPUTokenizer** d_tok) {
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(d_tok), sizeof(GPUTokenizer));
    if (e != cudaSuccess) return e;
    return tokenizer_init_gpu(*d_tok, h_tok);
}

// tokenizer_free_gpu (tokenizer_cuda.cu:274-285): the tables; the caller cudaFree's d_tok.
inline void tokenizer_free_gpu(GPUTokenizer* d_tok) {
    rbk_bpe* t = rubidium_tok_detail::handle(d_tok);
    if (!t) return;
    rbk_bpe_destroy(t);
    rubidium_tok_detail::registry().erase(d_tok);
}

// encode_batch (tokenizer_cuda.cu:287-332): rows of max_seq_len ids at d_output_tokens.
inline cudaError_t encode_batch(const GPUTokenizer* tok, const char** h_strings, int batch_size,
                                int* d_output_tokens, int* d_output_lengths, int max_seq_len,
                                cudaStream_t stream = 0) {
    rbk_bpe* t = rubidium_tok_detail::handle(tok);
    if (!t) return cudaErrorInvalidValue;
    return rubidium_tok_detail::to_cuda(rbk_bpe_encode_batch(t, h_strings, batch_size, d_output_tokens,
                                                             d_output_lengths, max_seq_len, stream));
}

// decode_batch (tokenizer_cuda.cu:334-348): as the reference, h_output_strings[0] is the
// device output buffer (batch_size rows of max_string_len bytes) and row b of the ids starts
// at b * d_input_lengths[b].
inline cudaError_t decode_batch(const GPUTokenizer* tok, const int* d_input_tokens, const int* d_input_lengths,
                                int batch_size, char** h_output_strings, int max_string_len,
                                cudaStream_t stream = 0) {
    rbk_bpe* t = rubidium_tok_detail::handle(tok);
    if (!t || !h_output_strings) return cudaErrorInvalidValue;
    return rubidium_tok_detail::to_cuda(rbk_bpe_decode_batch(t, d_input_tokens, 0, d_input_lengths, batch_size,
                                                             h_output_strings[0], max_string_len, nullptr,
                                                             stream));
}

// encode_string (tokenizer_cuda.cu:350-366).  The text up to its first NUL, cut to
// max_seq_len - 1 bytes; an empty vector on an error.
inline std::vector<int> encode_string(const GPUTokenizer* d_tok, const std::string& text,
                                      int max_seq_len = MAX_SEQ_LEN) {
    rbk_bpe* t = rubidium_tok_detail::handle(d_tok);
    if (!t || max_seq_len < 2) return {};
    const int n = (int)strlen(text.c_str());
    uint8_t* d_bytes = nullptr;
    int64_t* d_off = nullptr;
    int *d_len = nullptr, *d_out = nullptr, *d_out_len = nullptr;
    const int64_t zero = 0;
    std::vector<int> tokens;
    if (cudaMalloc(&d_bytes, std::max(n, 1)) == cudaSuccess && cudaMalloc(&d_off, sizeof(int64_t)) == cudaSuccess &&
        cudaMalloc(&d_len, sizeof(int)) == cudaSuccess && cudaMalloc(&d_out, sizeof(int) * max_seq_len) == cudaSuccess &&
        cudaMalloc(&d_out_len, sizeof(int)) == cudaSuccess &&
        cudaMemcpy(d_bytes, text.data(), n, cudaMemcpyHostToDevice) == cudaSuccess &&
        cudaMemcpy(d_off, &zero, sizeof(zero), cudaMemcpyHostToDevice) == cudaSuccess &&
        cudaMemcpy(d_len, &n, sizeof(n), cudaMemcpyHostToDevice) == cudaSuccess &&
        rbk_bpe_encode(t, d_bytes, d_off, d_len, 1, d_out, d_out_len, max_seq_len, nullptr, nullptr) == RBK_OK) {
        int length = 0;
        if (cudaMemcpy(&length, d_out_len, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess) {
            tokens.resize(length);
            if (cudaMemcpy(tokens.data(), d_out, sizeof(int) * length, cudaMemcpyDeviceToHost) != cudaSuccess)
                tokens.clear();
        }
    }
    cudaFree(d_bytes);
    cudaFree(d_off);
    cudaFree(d_len);
    cudaFree(d_out);
    cudaFree(d_out_len);
    return tokens;
}

// decode_tokens (tokenizer_cuda.cu:368-389): at most 1023 bytes, as the reference's buffer.
inline std::string decode_tokens(const GPUTokenizer* d_tok, const std::vector<int>& tokens) {
    rbk_bpe* t = rubidium_tok_detail::handle(d_tok);
    if (!t) return {};
    constexpr int kLen = 1024;
    int *d_in = nullptr, *d_n = nullptr;
    char* d_str = nullptr;
    const int n = (int)tokens.size();
    std::string out;
    if (cudaMalloc(&d_in, sizeof(int) * std::max(n, 1)) == cudaSuccess && cudaMalloc(&d_n, sizeof(int)) == cudaSuccess &&
        cudaMalloc(&d_str, kLen) == cudaSuccess &&
        cudaMemcpy(d_in, tokens.data(), sizeof(int) * n, cudaMemcpyHostToDevice) == cudaSuccess &&
        cudaMemcpy(d_n, &n, sizeof(n), cudaMemcpyHostToDevice) == cudaSuccess &&
        rbk_bpe_decode_batch(t, d_in, 0, d_n, 1, d_str, kLen, nullptr, nullptr) == RBK_OK) {
        char buf[kLen];
        if (cudaMemcpy(buf, d_str, kLen, cudaMemcpyDeviceToHost) == cudaSuccess) out.assign(buf, strnlen(buf, kLen));
    }
    cudaFree(d_in);
    cudaFree(d_n);
    cudaFree(d_str);
    return out;
}

inline void tokenizer_print_stats(const HostTokenizer& tok) {
    printf("Vocab size: %d\n", tok.vocab_size);
    printf("Merges: %zu\n", tok.merges.size());
    printf("Unigram entries: %zu\n", tok.unigram_probs.size());
}

// Every string encodes and decodes back to itself (strings without NUL bytes, shorter than
// MAX_SEQ_LEN and 1024 bytes, whose ids all carry their strings in h_tok.inv_vocab).
inline bool tokenizer_validate_roundtrip(const HostTokenizer& h_tok, const GPUTokenizer* d_tok,
                                         const std::vector<std::string>& test_strings) {
    (void)h_tok;
    for (const auto& s : test_strings) {
        std::vector<int> ids = encode_string(d_tok, s, MAX_SEQ_LEN);
        if (ids.empty() || decode_tokens(d_tok, ids) != s) return false;
    }
    return true;
}
