// embed.cu — token + position embedding forward and backward.
//
// Forward fuses embedding_fp16_forward with the per-batch pos_emb scale_add of
// the reference (src/model.cu:246-248).  Backward scatters dx into the token
// table with FP32 vector reductions (red.global.add.v4.f32, as the reference's
// per-element atomicAdd, src/cuda_kernels.cu:345-361) and sums pos_emb's
// gradient over the batch in a fixed order (the reference never computes it).
#include "common.cuh"

namespace rbk {
namespace {

__global__ void embed_fwd_kernel(half* __restrict__ x, const half* __restrict__ tok_emb,
                                 const half* __restrict__ pos_emb, const int* __restrict__ tokens, int N, int S,
                                 int D, int V) {
    const int nvec = D >> 3;
    const long total = (long)N * nvec;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int n = (int)(i / nvec), c = (int)(i % nvec);
        int t = __ldg(tokens + n);
        t = t < 0 ? 0 : (t >= V ? V - 1 : t);
        float a[8], b[8];
        h8_to_f(__ldg(reinterpret_cast<const uint4*>(tok_emb + (size_t)t * D) + c), a);
        h8_to_f(__ldg(reinterpret_cast<const uint4*>(pos_emb + (size_t)(n % S) * D) + c), b);
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] += b[j];
        reinterpret_cast<uint4*>(x + (size_t)n * D)[c] = f_to_h8(a);
    }
}

__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

__global__ void embed_tok_bwd_kernel(float* __restrict__ dtok, const half* __restrict__ dx,
                                     const int* __restrict__ tokens, int N, int D, int V) {
    const int nvec = D >> 3;
    const long total = (long)N * nvec;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int n = (int)(i / nvec), c = (int)(i % nvec);
        const int t = __ldg(tokens + n);
        if (t < 0 || t >= V) continue;
        float a[8];
        h8_to_f(__ldg(reinterpret_cast<const uint4*>(dx + (size_t)n * D) + c), a);
        float* dst = dtok + (size_t)t * D + 8 * c;
        red_add_v4(dst, a[0], a[1], a[2], a[3]);
        red_add_v4(dst + 4, a[4], a[5], a[6], a[7]);
    }
}

__global__ void embed_pos_bwd_kernel(float* __restrict__ dpos, const half* __restrict__ dx, int B, int S, int D) {
    const int nvec = D >> 3;
    const long total = (long)S * nvec;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int s = (int)(i / nvec), c = (int)(i % nvec);
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int b = 0; b < B; ++b) {
            float a[8];
            h8_to_f(__ldg(reinterpret_cast<const uint4*>(dx + ((size_t)b * S + s) * D) + c), a);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] += a[j];
        }
        float4* dst = reinterpret_cast<float4*>(dpos + (size_t)s * D + 8 * c);
        float4 u = dst[0], v = dst[1];
        u.x += acc[0]; u.y += acc[1]; u.z += acc[2]; u.w += acc[3];
        v.x += acc[4]; v.y += acc[5]; v.z += acc[6]; v.w += acc[7];
        dst[0] = u;
        dst[1] = v;
    }
}

int grid_for(long work, int num_sms) {
    long g = (work + 255) / 256;
    long cap = (long)num_sms * 8;
    return (int)(g < cap ? (g > 0 ? g : 1) : cap);
}

}  // namespace
}  // namespace rbk

using namespace rbk;

extern "C" {

int rbk_embed_fwd(rbk_ctx* ctx, void* x, const void* tok_emb, const void* pos_emb, const int* tokens, int B, int S,
                  int D, int V, void* stream) {
    RBK_REQUIRE(ctx && x && tok_emb && pos_emb && tokens, "rbk_embed_fwd: null pointer");
    RBK_REQUIRE(B > 0 && S > 0 && D > 0 && D % 8 == 0 && V > 0, "rbk_embed_fwd: bad shape");
    RBK_REQUIRE(aligned16(x) && aligned16(tok_emb) && aligned16(pos_emb), "rbk_embed_fwd: 16-byte alignment");
    const int N = B * S;
    embed_fwd_kernel<<<grid_for((long)N * (D / 8), ctx->num_sms), 256, 0, as_stream(stream)>>>(
        (half*)x, (const half*)tok_emb, (const half*)pos_emb, tokens, N, S, D, V);
    RBK_LAUNCHED("embed_fwd_kernel");
    return RBK_OK;
}

int rbk_embed_bwd(rbk_ctx* ctx, float* dtok, float* dpos, const void* dx, const int* tokens, int B, int S, int D,
                  int V, void* stream) {
    RBK_REQUIRE(ctx && dx && tokens, "rbk_embed_bwd: null pointer");
    RBK_REQUIRE(B > 0 && S > 0 && D > 0 && D % 8 == 0 && V > 0, "rbk_embed_bwd: bad shape");
    RBK_REQUIRE(aligned16(dx) && (!dtok || aligned16(dtok)) && (!dpos || aligned16(dpos)),
                "rbk_embed_bwd: 16-byte alignment");
    const int N = B * S;
    cudaStream_t st = as_stream(stream);
    ProfScope prof(ctx, st, kCatEmbed, (double)N * D * (2.0 + 8.0));
    if (dtok) {
        embed_tok_bwd_kernel<<<grid_for((long)N * (D / 8), ctx->num_sms), 256, 0, st>>>(dtok, (const half*)dx,
                                                                                       tokens, N, D, V);
        RBK_LAUNCHED("embed_tok_bwd_kernel");
    }
    if (dpos) {
        embed_pos_bwd_kernel<<<grid_for((long)S * (D / 8), ctx->num_sms), 256, 0, st>>>(dpos, (const half*)dx, B,
                                                                                       S, D);
        RBK_LAUNCHED("embed_pos_bwd_kernel");
    }
    return RBK_OK;
}

}  // extern "C"
