// embed.cu — token + position embedding forward and backward.
//
// Forward fuses embedding_fp16_forward with the per-batch pos_emb scale_add of
// the reference (src/model.cu:246-248).  Backward: the reference scatters dx
// into the token table with one atomicAdd per element (src/cuda_kernels.cu:
// 345-361), whose summation order changes from run to run; so does the default
// path here (16-byte vector reductions).  In deterministic mode the (token,
// position) pairs are sorted first and each distinct token's rows are summed in
// position order by one warp, so the token gradient is bitwise reproducible (up
// to 32768 positions per call).  pos_emb's gradient (which the reference never
// computes) is summed over the batch in a fixed order in both modes.
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

// ---- deterministic token gradient: sort (token, position) keys, then one warp per distinct token
// sums its rows in position order and adds the sum to its table row (one writer per row, no
// atomics), so repeated backwards give bit-identical gradients.
constexpr int kSortIdxBits = 15;                    // positions < 32768
constexpr int kSortMaxN = 1 << kSortIdxBits;
constexpr int kSortThreads = 1024;

// One CTA: keys = token << 15 | position (invalid tokens sort last as 0xFFFFFFFF), bitonic sort of
// the next power of two >= N keys in shared memory, sorted keys out.
__global__ void __launch_bounds__(kSortThreads) embed_sort_kernel(uint32_t* __restrict__ keys_out,
                                                                  const int* __restrict__ tokens, int N, int V,
                                                                  int P) {
    extern __shared__ uint32_t kk[];
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        uint32_t k = 0xFFFFFFFFu;
        if (i < N) {
            const int t = __ldg(tokens + i);
            if (t >= 0 && t < V) k = ((uint32_t)t << kSortIdxBits) | (uint32_t)i;
        }
        kk[i] = k;
    }
    __syncthreads();
    for (int size = 2; size <= P; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int t = threadIdx.x; t < (P >> 1); t += blockDim.x) {
                const int i = 2 * t - (t & (stride - 1));            // lower element of the pair
                const int j = i + stride;
                const bool up = (i & size) == 0;
                const uint32_t a = kk[i], b = kk[j];
                if ((a > b) == up) { kk[i] = b; kk[j] = a; }
            }
            __syncthreads();
        }
    }
    for (int i = threadIdx.x; i < N; i += blockDim.x) keys_out[i] = kk[i];
}

// Warp w starts at sorted position w; only the first position of each token's run does work.
__global__ void embed_tok_bwd_sorted_kernel(float* __restrict__ dtok, const half* __restrict__ dx,
                                            const uint32_t* __restrict__ keys, int N, int D) {
    const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (w >= N) return;
    const uint32_t k = __ldg(keys + w);
    if (k == 0xFFFFFFFFu) return;
    const uint32_t tok = k >> kSortIdxBits;
    if (w > 0 && (__ldg(keys + w - 1) >> kSortIdxBits) == tok) return;
    int end = w + 1;
    while (end < N && (__ldg(keys + end) >> kSortIdxBits) == tok && __ldg(keys + end) != 0xFFFFFFFFu) ++end;
    const int nvec = D >> 3;
    for (int c0 = 0; c0 < nvec; c0 += 32) {         // 256 columns per pass: one 16-byte piece per lane
        const int c = c0 + lane;
        if (c >= nvec) break;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int q = w; q < end; ++q) {             // positions in ascending order
            const int i = (int)(__ldg(keys + q) & (kSortMaxN - 1));
            float a[8];
            h8_to_f(__ldg(reinterpret_cast<const uint4*>(dx + (size_t)i * D) + c), a);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] += a[j];
        }
        float4* dst = reinterpret_cast<float4*>(dtok + (size_t)tok * D + 8 * c);
        float4 u = dst[0], v = dst[1];
        u.x += acc[0]; u.y += acc[1]; u.z += acc[2]; u.w += acc[3];
        v.x += acc[4]; v.y += acc[5]; v.z += acc[6]; v.w += acc[7];
        dst[0] = u;
        dst[1] = v;
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
    if (dtok && ctx->deterministic && N <= kSortMaxN && V <= (1 << (32 - kSortIdxBits)) - 1) {
        // deterministic mode: sort (token, position), then one writer per table row
        int P = 1;
        while (P < N) P <<= 1;
        void* ws;
        RBK_TRY(ctx_scratch(ctx, sizeof(uint32_t) * (size_t)N, &ws));
        const size_t smem = sizeof(uint32_t) * (size_t)P;
        if (smem > 48 * 1024)
            RBK_CUDA(cudaFuncSetAttribute(embed_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        embed_sort_kernel<<<1, kSortThreads, smem, st>>>((uint32_t*)ws, tokens, N, V, P);
        RBK_LAUNCHED("embed_sort_kernel");
        embed_tok_bwd_sorted_kernel<<<(N * 32 + 255) / 256, 256, 0, st>>>(dtok, (const half*)dx,
                                                                          (const uint32_t*)ws, N, D);
        RBK_LAUNCHED("embed_tok_bwd_sorted_kernel");
    } else if (dtok) {
        // vector reductions into the table (summation order not fixed; about 4x faster than sorting)
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
