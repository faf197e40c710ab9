// softmax.cu — row softmax backward over materialised attention probabilities
// (HBM-bound): dS = P * (dP - <dP, P>) per row, as softmax_fp16_bwd_kernel /
// cpuops::softmax_backward (reference src/cuda_kernels.cu:440-470,
// src/cpu_mat.h:190-200).  One warp per row; with `causal` the row i only
// touches columns 0..i, so only the lower triangle is read or written.
#include "common.cuh"

namespace rbk {
namespace {

template <int NV, bool kCausal>
__global__ void __launch_bounds__(256) attn_softmax_bwd_kernel(half* __restrict__ dS, const half* __restrict__ P,
                                                               const half* __restrict__ dP, long rows, int T) {
    const int lane = threadIdx.x & 31;
    const long warps = (long)gridDim.x * (blockDim.x >> 5);
    const int nvec = T >> 3;
    for (long r = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const int i = (int)(r % T);
        const int last = kCausal ? i : T - 1;          // last valid column
        const uint4* pr = reinterpret_cast<const uint4*>(P + (size_t)r * T);
        const uint4* dr = reinterpret_cast<const uint4*>(dP + (size_t)r * T);
        uint4 pv[NV], dv[NV];
        float dot = 0.0f;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int c = lane + 32 * k;
            const bool ok = c < nvec && 8 * c <= last;
            pv[k] = ok ? __ldg(pr + c) : make_uint4(0, 0, 0, 0);
            dv[k] = ok ? __ldg(dr + c) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int c = lane + 32 * k;
            if (c < nvec && 8 * c <= last) {
                float p[8], d[8];
                h8_to_f(pv[k], p);
                h8_to_f(dv[k], d);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (8 * c + j <= last) dot += p[j] * d[j];
            }
        }
        dot = warp_sum(dot);
        uint4* out = reinterpret_cast<uint4*>(dS + (size_t)r * T);
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const int c = lane + 32 * k;
            if (c < nvec && 8 * c <= last) {
                float p[8], d[8], o[8];
                h8_to_f(pv[k], p);
                h8_to_f(dv[k], d);
#pragma unroll
                for (int j = 0; j < 8; ++j) o[j] = p[j] * (d[j] - dot);
                if (8 * c + 7 <= last) {
                    out[c] = f_to_h8(o);
                } else {
                    half* o1 = dS + (size_t)r * T + 8 * c;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (8 * c + j <= last) o1[j] = __float2half_rn(o[j]);
                }
            }
        }
    }
}

template <int NV>
void launch(bool causal, int grid, cudaStream_t st, half* dS, const half* P, const half* dP, long rows, int T) {
    if (causal)
        attn_softmax_bwd_kernel<NV, true><<<grid, 256, 0, st>>>(dS, P, dP, rows, T);
    else
        attn_softmax_bwd_kernel<NV, false><<<grid, 256, 0, st>>>(dS, P, dP, rows, T);
}

}  // namespace
}  // namespace rbk

using namespace rbk;

extern "C" int rbk_attn_softmax_bwd(rbk_ctx* ctx, void* dS, const void* P, const void* dP, int nmat, int T,
                                    int causal, void* stream) {
    RBK_REQUIRE(ctx && dS && P && dP, "rbk_attn_softmax_bwd: null pointer");
    RBK_REQUIRE(nmat > 0 && T > 0 && T % 8 == 0 && T <= 8192, "rbk_attn_softmax_bwd: need T %% 8 == 0, T <= 8192");
    RBK_REQUIRE(aligned16(dS) && aligned16(P) && aligned16(dP), "rbk_attn_softmax_bwd: 16-byte alignment");
    const long rows = (long)nmat * T;
    const int nv = (T / 8 + 31) / 32;
    long g = (rows + 7) / 8;
    const long cap = (long)ctx->num_sms * 8;
    const int grid = (int)(g < cap ? g : cap);
    cudaStream_t st = as_stream(stream);
    const double elems = causal ? (double)nmat * T * (T + 1) / 2.0 : (double)nmat * T * T;
    ProfScope prof(ctx, st, kCatOther, 6.0 * elems);
    auto o = (half*)dS;
    auto p = (const half*)P;
    auto d = (const half*)dP;
    const bool c = causal != 0;
    switch (nv) {
        case 1: launch<1>(c, grid, st, o, p, d, rows, T); break;
        case 2: launch<2>(c, grid, st, o, p, d, rows, T); break;
        case 3: case 4: launch<4>(c, grid, st, o, p, d, rows, T); break;
        case 5: case 6: case 7: case 8: launch<8>(c, grid, st, o, p, d, rows, T); break;
        case 9: case 10: case 11: case 12: case 13: case 14: case 15: case 16:
            launch<16>(c, grid, st, o, p, d, rows, T); break;
        default: launch<32>(c, grid, st, o, p, d, rows, T); break;
    }
    RBK_LAUNCHED("attn_softmax_bwd_kernel");
    return RBK_OK;
}
