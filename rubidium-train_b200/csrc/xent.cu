// xent.cu — fused softmax-cross-entropy forward + backward (HBM-bound).
//
// One CTA owns a row: the row is read once into registers (16-byte vectors,
// kept as half2), reduced for its max and sum of exponentials, and the
// gradient (softmax - onehot) * scale is written from the same registers, in
// place if the caller wishes.  The reference reads the whole row twice per
// element (src/cuda_kernels.cu:533-551, O(N V^2)); cpuops does three passes
// (src/cpu_mat.h:220-236).  Per-row loss follows src/cpu_mat.h:213
// (-log(p_t + 1e-10)).
#include <cfloat>

#include "common.cuh"

namespace rbk {
namespace {

__device__ __forceinline__ float block_reduce_max(float v, float* sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_max(v);
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    float r = lane < nw ? sh[lane] : -FLT_MAX;
    r = warp_max(r);
    __syncthreads();
    return r;
}
__device__ __forceinline__ float block_reduce_sum(float v, float* sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    float r = lane < nw ? sh[lane] : 0.0f;
    r = warp_sum(r);
    __syncthreads();
    return r;
}

template <int E>
__global__ void __launch_bounds__(512) xent_kernel(half* dl, const half* lg, int ld, const int* __restrict__ tgt,
                                                   int N, int V, float scale, const float* __restrict__ dscale,
                                                   float* __restrict__ row_loss) {
    __shared__ float sh[32];
    const float gs = scale * (dscale ? __ldg(dscale) : 1.0f);
    const int nt = blockDim.x, tid = threadIdx.x;
    const half NEG = __float2half(-65504.0f);
    for (int row = blockIdx.x; row < N; row += gridDim.x) {
        const half* z = lg + (size_t)row * ld;
        uint4 raw[E];
        float mx = -FLT_MAX;
#pragma unroll
        for (int k = 0; k < E; ++k) {
            const int c = tid + k * nt;
            const int col = 8 * c;
            if (col + 8 <= V) {
                raw[k] = *reinterpret_cast<const uint4*>(z + col);
            } else {
                half h[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) h[j] = (col + j < V) ? z[col + j] : NEG;
                raw[k] = *reinterpret_cast<uint4*>(h);
            }
            if (col < V) {
                const __half2* h2 = reinterpret_cast<const __half2*>(&raw[k]);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float2 f = __half22float2(h2[j]);
                    mx = fmaxf(mx, fmaxf(f.x, f.y));
                }
            }
        }
        mx = block_reduce_max(mx, sh);
        // exponentials kept as float pairs would double the registers; keep the
        // raw logits and recompute exp in the write pass only where needed.
        float s = 0.0f;
#pragma unroll
        for (int k = 0; k < E; ++k) {
            const int col = 8 * (tid + k * nt);
            if (col < V) {
                const __half2* h2 = reinterpret_cast<const __half2*>(&raw[k]);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float2 f = __half22float2(h2[j]);
                    const float e0 = (col + 2 * j < V) ? __expf(f.x - mx) : 0.0f;
                    const float e1 = (col + 2 * j + 1 < V) ? __expf(f.y - mx) : 0.0f;
                    s += e0 + e1;
                }
            }
        }
        s = block_reduce_sum(s, sh);
        const float inv = 1.0f / s;
        const int t = __ldg(tgt + row);
        const bool tvalid = t >= 0 && t < V;
        if (row_loss && tid == 0) {
            float l = __int_as_float(0x7fc00000);   // NaN for an invalid target
            if (tvalid) l = -logf(__expf(__half2float(z[t]) - mx) * inv + 1e-10f);
            row_loss[row] = l;
        }
        if (!dl) continue;   // loss-only mode
        const float g = tvalid ? gs : 0.0f;
        half* d = dl + (size_t)row * ld;
#pragma unroll
        for (int k = 0; k < E; ++k) {
            const int col = 8 * (tid + k * nt);
            if (col >= V) continue;
            const __half2* h2 = reinterpret_cast<const __half2*>(&raw[k]);
            float o[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float2 f = __half22float2(h2[j]);
                o[2 * j] = (__expf(f.x - mx) * inv - (col + 2 * j == t ? 1.0f : 0.0f)) * g;
                o[2 * j + 1] = (__expf(f.y - mx) * inv - (col + 2 * j + 1 == t ? 1.0f : 0.0f)) * g;
            }
            if (col + 8 <= V) {
                *reinterpret_cast<uint4*>(d + col) = f_to_h8(o);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (col + j < V) d[col + j] = __float2half_rn(o[j]);
            }
        }
    }
}

template <int E>
void launch(int grid, int nt, cudaStream_t st, half* dl, const half* lg, int ld, const int* tgt, int N, int V,
            float scale, const float* dscale, float* row_loss) {
    xent_kernel<E><<<grid, nt, 0, st>>>(dl, lg, ld, tgt, N, V, scale, dscale, row_loss);
}

}  // namespace
}  // namespace rbk

using namespace rbk;

extern "C" int rbk_softmax_xent_bwd(rbk_ctx* ctx, void* dlogits, const void* logits, int ld, const int* targets,
                                    int N, int V, float scale, const float* dscale, float* row_loss, void* stream) {
    RBK_REQUIRE(ctx && logits && targets && (dlogits || row_loss), "rbk_softmax_xent_bwd: null pointer");
    RBK_REQUIRE(N > 0 && V > 0 && V <= 65536 && ld >= V && ld % 8 == 0,
                "rbk_softmax_xent_bwd: need 0 < V <= 65536, ld >= V, ld %% 8 == 0 (V=%d ld=%d)", V, ld);
    RBK_REQUIRE((!dlogits || aligned16(dlogits)) && aligned16(logits),
                "rbk_softmax_xent_bwd: tensors must be 16-byte aligned");
    int nt = ((V + 63) / 64 + 31) / 32 * 32;
    nt = nt < 128 ? 128 : nt > 512 ? 512 : nt;
    const int e = (V + 8 * nt - 1) / (8 * nt);
    const int per_sm = 2048 / nt;
    int grid = ctx->num_sms * per_sm;
    if (grid > N) grid = N;
    cudaStream_t st = as_stream(stream);
    ProfScope prof(ctx, st, kCatXent,
                   (double)N * V * (dlogits ? 4.0 : 2.0) + 4.0 * N + (row_loss ? 4.0 * N : 0.0));
    auto DL = (half*)dlogits;
    auto LG = (const half*)logits;
    if (e <= 1) launch<1>(grid, nt, st, DL, LG, ld, targets, N, V, scale, dscale, row_loss);
    else if (e <= 2) launch<2>(grid, nt, st, DL, LG, ld, targets, N, V, scale, dscale, row_loss);
    else if (e <= 4) launch<4>(grid, nt, st, DL, LG, ld, targets, N, V, scale, dscale, row_loss);
    else if (e <= 8) launch<8>(grid, nt, st, DL, LG, ld, targets, N, V, scale, dscale, row_loss);
    else if (e <= 12) launch<12>(grid, nt, st, DL, LG, ld, targets, N, V, scale, dscale, row_loss);
    else launch<16>(grid, nt, st, DL, LG, ld, targets, N, V, scale, dscale, row_loss);
    RBK_LAUNCHED("xent_kernel");
    return RBK_OK;
}
