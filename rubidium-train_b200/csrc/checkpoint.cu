// checkpoint.cu — model checkpoints: the reference's RBN2 file with its
// device-pointer I/O fixed, plus the optimizer and loss-scaler state.
//
// The reference's save/load (src/model.cu:585-679) writes "RBN2", the six
// config ints, a 256-entry character map and the FP16 weights, but hands
// device pointers straight to fwrite / fread (it never copies them to or from
// the host), and it drops the FP32 masters, the Adam moments and the loss
// scaler, so a resumed run restarts Adam and the scale schedule.  Here:
//
//   "RBN2" | V T D H L FF (int32) | char map [256] (int32) |
//   FP16 weights, reference tensor order (below)            <- the reference's file
//   "RBKX" | version (int32) | element count (int64) | rbk_scaler (32 bytes) |
//   FP32 masters | Adam m | Adam v, each in the same tensor order
//
// Reference tensor order (src/model.cu:605-619): token_emb, pos_emb; per layer
// ln1_w ln1_b ln2_w ln2_b wq bq wk bk wv bv wo bo w1 b1 w2 b2; ln_f_w ln_f_b
// lm_w lm_b.  Every tensor is written as rows * cols elements, [out, in]
// row-major, without the arena's 64-element padding.  A file without the
// extension block (the reference's own layout) still loads: masters become the
// FP16 weights widened to FP32 (convert_weights_fp16_to_fp32, src/model.cu:672),
// the moments are zero and the scaler restarts.  Gradients are zeroed on load.
#include <cstdio>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "model.h"

namespace rbk {
namespace {

constexpr int kCkptVersion = 1;

// Arena indices in the reference's file order.
std::vector<int> file_order(const rbk_config& c) {
    static const int per_layer[RBK_N_LAYER_TENSORS] = {RBK_LN1_W, RBK_LN1_B, RBK_LN2_W, RBK_LN2_B, RBK_WQ, RBK_BQ,
                                                       RBK_WK,    RBK_BK,    RBK_WV,    RBK_BV,    RBK_WO, RBK_BO,
                                                       RBK_W1,    RBK_B1,    RBK_W2,    RBK_B2};
    std::vector<int> o;
    o.push_back(RBK_TOK_EMB);
    o.push_back(RBK_POS_EMB);
    for (int l = 0; l < c.L; ++l)
        for (int j = 0; j < RBK_N_LAYER_TENSORS; ++j) o.push_back(rbk_layer_tensor(l, per_layer[j]));
    for (int j = 0; j < RBK_N_TAIL_GLOBALS; ++j) o.push_back(rbk_tail_tensor(&c, j));
    return o;
}

struct File {
    FILE* f = nullptr;
    ~File() {
        if (f) fclose(f);
    }
};

int io_fail(const char* what, const char* path) {
    set_error("%s: %s", what, path);
    return RBK_ERR_IO;
}

// Copy one family's tensors (element size es) between the device arena and the file, tensor by
// tensor through a host buffer sized for the largest tensor.
int write_family(FILE* f, const rbk_model* m, const std::vector<int>& order, const void* dev, size_t es,
                 std::vector<char>& buf, const char* path) {
    for (int i : order) {
        const rbk_tensor& t = m->tab[i];
        const size_t bytes = (size_t)(t.rows * t.cols) * es;
        RBK_CUDA(cudaMemcpy(buf.data(), (const char*)dev + (size_t)t.offset * es, bytes, cudaMemcpyDeviceToHost));
        if (fwrite(buf.data(), 1, bytes, f) != bytes) return io_fail("rbk_model_save: write failed", path);
    }
    return RBK_OK;
}

int read_family(FILE* f, const rbk_model* m, const std::vector<int>& order, void* dev, size_t es,
                std::vector<char>& buf, const char* path) {
    for (int i : order) {
        const rbk_tensor& t = m->tab[i];
        const size_t bytes = (size_t)(t.rows * t.cols) * es;
        if (fread(buf.data(), 1, bytes, f) != bytes) return io_fail("rbk_model_load: file is truncated", path);
        RBK_CUDA(cudaMemcpy((char*)dev + (size_t)t.offset * es, buf.data(), bytes, cudaMemcpyHostToDevice));
    }
    return RBK_OK;
}

size_t largest_tensor(const rbk_model* m) {
    size_t mx = 0;
    for (const rbk_tensor& t : m->tab) mx = (size_t)(t.rows * t.cols) > mx ? (size_t)(t.rows * t.cols) : mx;
    return mx;
}

int64_t file_elems(const rbk_model* m) {
    int64_t s = 0;
    for (const rbk_tensor& t : m->tab) s += t.rows * t.cols;
    return s;
}

}  // namespace
}  // namespace rbk

using namespace rbk;

extern "C" int rbk_model_save(rbk_model* m, const char* path, const int* char_map, void* stream) {
    RBK_REQUIRE(m && path, "rbk_model_save: null pointer");
    RBK_CUDA(cudaSetDevice(m->ctx->device));
    RBK_TRY(dp_gather_state(m, as_stream(stream)));       // sharded optimizer: whole masters / moments
    RBK_TRY(dp_wait_weights(m, -1, as_stream(stream)));
    RBK_CUDA(cudaStreamSynchronize(as_stream(stream)));   // the last optimizer step has landed
    File fh;
    fh.f = fopen(path, "wb");
    if (!fh.f) return io_fail("rbk_model_save: cannot open for writing", path);
    FILE* f = fh.f;
    const rbk_config& c = m->lay;
    const int hdr[6] = {c.V, c.T, c.D, c.H, c.L, c.FF};
    int map[256] = {};
    if (char_map) std::memcpy(map, char_map, sizeof(map));
    if (fwrite("RBN2", 1, 4, f) != 4 || fwrite(hdr, sizeof(int), 6, f) != 6 || fwrite(map, sizeof(int), 256, f) != 256)
        return io_fail("rbk_model_save: write failed", path);
    const std::vector<int> order = file_order(c);
    std::vector<char> buf(largest_tensor(m) * sizeof(float));
    RBK_TRY(write_family(f, m, order, m->p16, sizeof(half), buf, path));
    // extension block: optimizer and scaler state
    rbk_scaler sc;
    RBK_CUDA(cudaMemcpy(&sc, m->scaler, sizeof(sc), cudaMemcpyDeviceToHost));
    const int ver = kCkptVersion;
    const int64_t ne = file_elems(m);
    if (fwrite("RBKX", 1, 4, f) != 4 || fwrite(&ver, sizeof(int), 1, f) != 1 || fwrite(&ne, sizeof(ne), 1, f) != 1 ||
        fwrite(&sc, sizeof(sc), 1, f) != 1)
        return io_fail("rbk_model_save: write failed", path);
    RBK_TRY(write_family(f, m, order, m->p32, sizeof(float), buf, path));
    RBK_TRY(write_family(f, m, order, m->m, sizeof(float), buf, path));
    RBK_TRY(write_family(f, m, order, m->v, sizeof(float), buf, path));
    if (fflush(f) != 0) return io_fail("rbk_model_save: write failed", path);
    return RBK_OK;
}

extern "C" int rbk_model_load(rbk_model* m, const char* path, int* char_map_out, void* stream) {
    RBK_REQUIRE(m && path, "rbk_model_load: null pointer");
    RBK_CUDA(cudaSetDevice(m->ctx->device));
    cudaStream_t st = as_stream(stream);
    RBK_TRY(dp_wait_weights(m, -1, st));                  // no all-gather still writes the weights
    RBK_CUDA(cudaStreamSynchronize(st));                  // no kernel still reads the arenas
    File fh;
    fh.f = fopen(path, "rb");
    if (!fh.f) return io_fail("rbk_model_load: cannot open", path);
    FILE* f = fh.f;
    char magic[4];
    int hdr[6], map[256];
    if (fread(magic, 1, 4, f) != 4 || fread(hdr, sizeof(int), 6, f) != 6 || fread(map, sizeof(int), 256, f) != 256)
        return io_fail("rbk_model_load: file is truncated", path);
    RBK_REQUIRE(std::memcmp(magic, "RBN2", 4) == 0, "rbk_model_load: %s is not an RBN2 checkpoint", path);
    const rbk_config& c = m->lay;
    RBK_REQUIRE(hdr[0] == c.V && hdr[1] == c.T && hdr[2] == c.D && hdr[3] == c.H && hdr[4] == c.L && hdr[5] == c.FF,
                "rbk_model_load: %s holds V=%d T=%d D=%d H=%d L=%d FF=%d, the model is V=%d T=%d D=%d H=%d L=%d FF=%d",
                path, hdr[0], hdr[1], hdr[2], hdr[3], hdr[4], hdr[5], c.V, c.T, c.D, c.H, c.L, c.FF);
    if (char_map_out) std::memcpy(char_map_out, map, sizeof(map));
    const std::vector<int> order = file_order(c);
    std::vector<char> buf(largest_tensor(m) * sizeof(float));
    RBK_TRY(read_family(f, m, order, m->p16, sizeof(half), buf, path));
    RBK_CUDA(cudaMemset(m->grad, 0, sizeof(float) * m->n));

    char xm[4];
    const size_t got = fread(xm, 1, 4, f);
    if (got == 0 && feof(f)) {
        // the reference's layout: widen the FP16 weights into the masters, fresh optimizer state
        std::vector<half> h16;
        std::vector<float> h32;
        for (int i : order) {
            const rbk_tensor& t = m->tab[i];
            const size_t n = (size_t)(t.rows * t.cols);
            h16.resize(n);
            h32.resize(n);
            RBK_CUDA(cudaMemcpy(h16.data(), m->p16 + t.offset, n * sizeof(half), cudaMemcpyDeviceToHost));
            for (size_t k = 0; k < n; ++k) h32[k] = __half2float(h16[k]);
            RBK_CUDA(cudaMemcpy(m->p32 + t.offset, h32.data(), n * sizeof(float), cudaMemcpyHostToDevice));
        }
        RBK_CUDA(cudaMemset(m->m, 0, sizeof(float) * m->n));
        RBK_CUDA(cudaMemset(m->v, 0, sizeof(float) * m->n));
        rbk_scaler sc = {};
        sc.scale = m->opts.init_loss_scale > 0 ? m->opts.init_loss_scale : 65536.0f;
        sc.interval = m->opts.growth_interval > 0 ? m->opts.growth_interval : 2000;
        RBK_CUDA(cudaMemcpy(m->scaler, &sc, sizeof(sc), cudaMemcpyHostToDevice));
        m->dp.masters_partial = false;
        return RBK_OK;
    }
    RBK_REQUIRE(got == 4 && std::memcmp(xm, "RBKX", 4) == 0,
                "rbk_model_load: %s has unknown data after the FP16 weights", path);
    int ver = 0;
    int64_t ne = 0;
    rbk_scaler sc;
    if (fread(&ver, sizeof(int), 1, f) != 1 || fread(&ne, sizeof(ne), 1, f) != 1 || fread(&sc, sizeof(sc), 1, f) != 1)
        return io_fail("rbk_model_load: file is truncated", path);
    RBK_REQUIRE(ver == kCkptVersion, "rbk_model_load: %s has extension version %d (this library reads %d)", path,
                ver, kCkptVersion);
    RBK_REQUIRE(ne == file_elems(m), "rbk_model_load: %s holds %lld elements per family, the model %lld", path,
                (long long)ne, (long long)file_elems(m));
    RBK_TRY(read_family(f, m, order, m->p32, sizeof(float), buf, path));
    RBK_TRY(read_family(f, m, order, m->m, sizeof(float), buf, path));
    RBK_TRY(read_family(f, m, order, m->v, sizeof(float), buf, path));
    sc.status = 0;
    RBK_CUDA(cudaMemcpy(m->scaler, &sc, sizeof(sc), cudaMemcpyHostToDevice));
    m->dp.masters_partial = false;                        // every rank holds the whole state again
    return RBK_OK;
}
