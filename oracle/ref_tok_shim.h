// ref_tok_shim.h — lets g++ compile the reference's GPU tokenizer kernels
// (src/tokenizer_cuda.cu:17-203: fnv1a_hash, vocab_lookup, find_merge,
// encode_kernel, decode_kernel) as plain host code, so that they run on the
// CPU as the pin of the tokenizer oracle.  TEST INFRASTRUCTURE ONLY
// (oracle/Makefile, target `ref`; output in oracle/_ref/, git-ignored).
//
// The reference header src/tokenizer_cuda.h does not compile as written: its
// PAD_ID..SEP_ID macros (:20-24) expand inside HostTokenizer's members of the
// same names (:102-106).  The kernel section needs only the device-side
// structs, so this header declares them itself with the reference's field
// names, types and order (tokenizer_cuda.h:31-88) and the reference header is
// never included.  The host-side table builders (HostTokenizer::build_*) are
// not compiled; ref_tok_shim.cpp lays the tables out as they do.
//
// The execution-space keywords become empty; threadIdx / blockIdx / blockDim
// become host globals that ref_tok_shim.cpp sets before each emulated thread;
// __syncthreads is a no-op.  That is exact for these two kernels:
// encode_kernel (tokenizer_cuda.cu:90-167) has every thread write its own
// byte's token before one barrier, after which thread 0 alone works, so the
// shim runs threads blockDim-1 .. 0 in turn and thread 0 sees every write;
// decode_kernel (tokenizer_cuda.cu:169-203) runs one thread per block.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstring>

#define __device__
#define __host__
#define __global__
#define __shared__

struct RefTokDim {
    unsigned x, y, z;
};
extern RefTokDim ref_tok_thread_idx, ref_tok_block_idx, ref_tok_block_dim;
#define threadIdx ref_tok_thread_idx
#define blockIdx ref_tok_block_idx
#define blockDim ref_tok_block_dim
#define __syncthreads() ((void)0)

struct VocabEntry {
    uint64_t key_hash;
    int token_id;
    uint16_t length;
    char string_data[32];
};

struct MergeTrieNode {
    int child[256];
    int merge_id;
    int token_id;
};

struct MergeRule {
    int first_id;
    int second_id;
    int result_id;
    int priority;
};

struct UnigramEntry {
    int token_id;
    float log_prob;
};

struct GPUTokenizer {
    VocabEntry* d_vocab_table;
    int vocab_table_size;
    int vocab_size;
    MergeTrieNode* d_merge_trie;
    int merge_trie_size;
    int num_merges;
    MergeRule* d_merge_rules;
    UnigramEntry* d_unigram_probs;
    int unigram_size;
    char* d_inv_vocab_strings;
    int* d_inv_vocab_offsets;
    int* d_inv_vocab_lengths;
    int pad_id, unk_id, bos_id, eos_id, sep_id;
    int max_token_len;
};

// the kernel section as a function set of its own (defined in the piped translation unit)
void encode_kernel(const GPUTokenizer* tok, const char* strings_data, const int* string_offsets,
                   const int* string_lengths, int batch_size, int* output_tokens, int* output_lengths,
                   int max_seq_len);
void decode_kernel(const GPUTokenizer* tok, const int* input_tokens, const int* input_lengths, int batch_size,
                   char* output_strings, int max_string_len);
