// Element-wise kernels of the OLMo-2 decoder around the attention layer, used
// by the full-model prefill (configuration 3).  All HBM-bound; one 256-thread
// CTA per token row of d_model = 2048 (8 elements per thread).
//
//   embed_gather_kernel   x = embed[ids]                 (OlmoModel.cpp:34-38)
//   residual_norm_kernel  x = x + RMSNorm(y) * g         (OlmoBlock.cpp:15-16, :18-19;
//                                                         RMSNorm.cpp:15-22)
//                         or, without a residual, x = RMSNorm(y) * g (final norm,
//                         OlmoModel.cpp:45); writes fp32 (the residual stream)
//                         and/or bf16 (the next GEMM's operand).
#pragma once
#include "dt_common.cuh"

namespace dt {
namespace model {

constexpr int kD = 2048;
constexpr int kThreads = 256;

__device__ __forceinline__ float row_sum_256(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kThreads / 32; ++i) t += red[i];
    return t;
}

__device__ __forceinline__ void store8_bf16(__nv_bfloat16* dst, const float (&v)[8]) {
    uint4 w;
    w.x = pack_bf16x2(v[0], v[1]);
    w.y = pack_bf16x2(v[2], v[3]);
    w.z = pack_bf16x2(v[4], v[5]);
    w.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(dst) = w;
}

// x[row] = embed[ids[row]] (fp32 and bf16 copies).  Ids >= vocab are rejected on
// the host before launch; the kernel clamps them anyway so no read leaves the table.
__global__ void __launch_bounds__(kThreads)
embed_gather_kernel(const unsigned* __restrict__ ids, const float* __restrict__ embed, int vocab,
                    float* __restrict__ x, __nv_bfloat16* __restrict__ xb) {
    const long long row = blockIdx.x;
    const unsigned id = min(ids[row], (unsigned)(vocab - 1));
    const float4* src = reinterpret_cast<const float4*>(embed + (long long)id * kD) + 2 * threadIdx.x;
    const float4 a = src[0], b = src[1];
    float4* dst = reinterpret_cast<float4*>(x + row * kD) + 2 * threadIdx.x;
    dst[0] = a;
    dst[1] = b;
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    store8_bf16(xb + row * kD + 8 * threadIdx.x, v);
}

// out = (residual ? x : 0) + y / sqrt(mean(y^2) + eps) * g, per row.
// x_out may alias x; either output may be null.
__global__ void __launch_bounds__(kThreads)
residual_norm_kernel(const float* __restrict__ x, const float* __restrict__ y, const float* __restrict__ g,
                     float* x_out, __nv_bfloat16* xb_out, float eps, int residual) {
    __shared__ float red[kThreads / 32];
    const long long row = blockIdx.x;
    const int c0 = 8 * threadIdx.x;
    const float4* yr = reinterpret_cast<const float4*>(y + row * kD + c0);
    const float4 a = yr[0], b = yr[1];
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += v[e] * v[e];
    ss = row_sum_256(ss, red);
    const float rms = sqrtf(ss / (float)kD + eps);
    const float4* gr = reinterpret_cast<const float4*>(g + c0);
    const float4 ga = gr[0], gb = gr[1];
    const float gv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
    float o[8];
    if (residual) {
        const float4* xr = reinterpret_cast<const float4*>(x + row * kD + c0);
        const float4 xa = xr[0], xbv = xr[1];
        const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xbv.x, xbv.y, xbv.z, xbv.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = xv[e] + v[e] / rms * gv[e];
    } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = v[e] / rms * gv[e];
    }
    if (x_out) {
        float4* d = reinterpret_cast<float4*>(x_out + row * kD + c0);
        d[0] = make_float4(o[0], o[1], o[2], o[3]);
        d[1] = make_float4(o[4], o[5], o[6], o[7]);
    }
    if (xb_out) store8_bf16(xb_out + row * kD + c0, o);
}

}  // namespace model
}  // namespace dt
