// tokenizer_calls.cpp — the GPU-tokenizer calls of the reference's LoRA trainer
// (src/fine_tune.cu:100-125,148-157,284-285) and the rest of src/tokenizer_cuda.h's API,
// written against the drop-in header under the reference's own name ("tokenizer_cuda.h"
// from include/rubidium/compat).  The reference's HostTokenizer::load_from_json loads
// nothing, so the tables come from a text file:
//   V M N
//   V lines: id's string in hex ("-" when empty)
//   M lines: first second merged-string-hex
//   N lines: input string in hex
// Output, one line each: "E <ids>" from encode_string, "D <hex>" from decode_tokens per input;
// "B <len> <ids>" per row of one encode_batch over all inputs (rows of 2048);
// "R <hex>" per row of decode_batch over those rows in the reference's layout; "V <0|1>"
// from tokenizer_validate_roundtrip.
//   usage: tokenizer_calls <tables file>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <string>
#include <vector>

#include "tokenizer_cuda.h"

static std::string unhex(const std::string& h) {
    if (h == "-") return {};
    std::string s;
    for (size_t i = 0; i + 1 < h.size(); i += 2) s.push_back((char)std::stoi(h.substr(i, 2), nullptr, 16));
    return s;
}

static std::string hex(const std::string& s) {
    static const char* d = "0123456789abcdef";
    std::string h;
    for (unsigned char c : s) {
        h.push_back(d[c >> 4]);
        h.push_back(d[c & 15]);
    }
    return h.empty() ? "-" : h;
}

int main(int argc, char** argv) {
    if (argc < 2) {
        fprintf(stderr, "usage: tokenizer_calls <tables file>\n");
        return 2;
    }
    std::ifstream f(argv[1]);
    int V = 0, M = 0, N = 0;
    f >> V >> M >> N;
    HostTokenizer h;
    if (h.load_from_json("tokenizer.json")) return 3;  // the reference's loader loads nothing
    for (int i = 0; i < V; ++i) {
        std::string x;
        f >> x;
        const std::string s = unhex(x);
        h.inv_vocab[i] = s;
        if (!s.empty()) h.vocab[s] = i;
    }
    h.vocab_size = V;
    for (int j = 0; j < M; ++j) {
        int a, b;
        std::string x;
        f >> a >> b >> x;
        h.merges.push_back({{a, b}, unhex(x)});
    }
    std::vector<std::string> inputs(N);
    for (auto& s : inputs) {
        std::string x;
        f >> x;
        s = unhex(x);
    }

    GPUTokenizer* d_tok = nullptr;
    if (tokenizer_copy_to_device(h, &d_tok) != cudaSuccess) {
        fprintf(stderr, "tokenizer_copy_to_device failed: %s\n", rbk_last_error());
        return 1;
    }
    // tokenize_instructions' loop (src/fine_tune.cu:108-120)
    for (const auto& s : inputs) {
        std::vector<int> ids = encode_string(d_tok, s, MAX_SEQ_LEN);
        printf("E");
        for (int t : ids) printf(" %d", t);
        printf("\nD %s\n", hex(decode_tokens(d_tok, ids)).c_str());
    }
    // encode_batch / decode_batch over the whole set
    const int ms = MAX_SEQ_LEN;
    std::vector<const char*> ptrs;
    for (const auto& s : inputs) ptrs.push_back(s.c_str());
    int *d_rows = nullptr, *d_lens = nullptr;
    cudaMalloc(&d_rows, sizeof(int) * ms * N);
    cudaMalloc(&d_lens, sizeof(int) * N);
    if (encode_batch(d_tok, ptrs.data(), N, d_rows, d_lens, ms) != cudaSuccess) {
        fprintf(stderr, "encode_batch failed: %s\n", rbk_last_error());
        return 1;
    }
    std::vector<int> rows((size_t)ms * N), lens(N);
    cudaMemcpy(rows.data(), d_rows, sizeof(int) * ms * N, cudaMemcpyDeviceToHost);
    cudaMemcpy(lens.data(), d_lens, sizeof(int) * N, cudaMemcpyDeviceToHost);
    std::vector<int> flat;  // the reference's decode layout: row b at b * lens[b]
    for (int b = 0; b < N; ++b) {
        printf("B %d", lens[b]);
        for (int i = 0; i < lens[b]; ++i) printf(" %d", rows[(size_t)b * ms + i]);
        printf("\n");
        flat.resize(std::max(flat.size(), (size_t)b * lens[b] + lens[b]));
        for (int i = 0; i < lens[b]; ++i) flat[(size_t)b * lens[b] + i] = rows[(size_t)b * ms + i];
    }
    const int msl = 4096;
    int* d_flat = nullptr;
    char* d_out = nullptr;
    cudaMalloc(&d_flat, sizeof(int) * std::max<size_t>(flat.size(), 1));
    cudaMalloc(&d_out, (size_t)msl * N);
    cudaMemcpy(d_flat, flat.data(), sizeof(int) * flat.size(), cudaMemcpyHostToDevice);
    char* outs[1] = {d_out};
    if (decode_batch(d_tok, d_flat, d_lens, N, outs, msl) != cudaSuccess) {
        fprintf(stderr, "decode_batch failed: %s\n", rbk_last_error());
        return 1;
    }
    std::vector<char> text((size_t)msl * N);
    cudaMemcpy(text.data(), d_out, text.size(), cudaMemcpyDeviceToHost);
    for (int b = 0; b < N; ++b) printf("R %s\n", hex(std::string(text.data() + (size_t)b * msl)).c_str());
    std::vector<std::string> short_inputs;
    for (const auto& s : inputs)
        if (s.size() < 1000) short_inputs.push_back(s);
    printf("V %d\n", tokenizer_validate_roundtrip(h, d_tok, short_inputs) ? 1 : 0);
    cudaFree(d_rows);
    cudaFree(d_lens);
    cudaFree(d_flat);
    cudaFree(d_out);
    tokenizer_free_gpu(d_tok);
    cudaFree(d_tok);  // src/fine_tune.cu:285
    return 0;
}
