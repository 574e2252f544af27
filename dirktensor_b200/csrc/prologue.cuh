// HBM-bound element-wise kernels of the attention hot path.
//
// cast_f32_bf16 : fp32 -> bf16 (same layout), for the projection input x and
//                 for raw fp32 Q/K/V handed to flash_attention_forward.
// qk_norm_rope  : the prologue between the QKV projection and attention:
//                 q = RoPE(RMSNorm_q(xWq^T)), k = RoPE(RMSNorm_k(xWk^T)),
//                 v = xWv^T, all written as bf16 in [B, T, H, D] layout.
//   RMSNorm follows RMSNorm.cpp:15-22 (rms = sqrt(mean(x^2) + eps) over the
//   whole d_model = 2048 row, i.e. across all heads; y = x / rms * g), RoPE
//   follows OlmoAttention.cpp:111-146 (rotate-half, position = t, tables from
//   OlmoAttention.cpp:18-36).  One CTA of 256 threads per token: thread i owns
//   head i/16 and the dims {4j..4j+3} U {64+4j..64+4j+3} (j = i%16) of q and k,
//   i.e. both members of its RoPE pairs, so RoPE needs no data exchange; the two
//   sums of squares are reduced across the CTA.
#pragma once
#include "dt_common.cuh"

namespace dt {
namespace elem {

// n4: number of float4 groups; each thread handles float4 groups grid-stride.
__global__ void cast_f32_bf16_kernel(const float4* __restrict__ src, uint2* __restrict__ dst, long long n4) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
         i += (long long)gridDim.x * blockDim.x) {
        const float4 v = src[i];
        uint2 w;
        w.x = pack_bf16x2(v.x, v.y);
        w.y = pack_bf16x2(v.z, v.w);
        dst[i] = w;
    }
}

// Three tensors in one launch (raw Q, K, V); blockIdx.y selects the tensor.
struct Cast3 {
    const float4* src[3];
    uint2* dst[3];
};
__global__ void cast3_f32_bf16_kernel(Cast3 a, long long n4) {
    const float4* __restrict__ src = a.src[blockIdx.y];
    uint2* __restrict__ dst = a.dst[blockIdx.y];
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
         i += (long long)gridDim.x * blockDim.x) {
        const float4 v = src[i];
        uint2 w;
        w.x = pack_bf16x2(v.x, v.y);
        w.y = pack_bf16x2(v.z, v.w);
        dst[i] = w;
    }
}

constexpr int kDModel = 2048;
constexpr int kHeadDim = 128;
constexpr int kPrologueThreads = 256;

struct PrologueParams {
    const float* q;       // [M, ld_in] rows of the projection output (q part)
    const float* k;
    const float* v;
    long long ld_in;      // elements between consecutive tokens
    const float* q_gain;  // [2048]
    const float* k_gain;  // [2048]
    const float* sin_t;   // [max_seq, 128]
    const float* cos_t;   // [max_seq, 128]
    __nv_bfloat16* qo;    // [M, 2048]
    __nv_bfloat16* ko;
    __nv_bfloat16* vo;
    int T;                // tokens per sequence: position of row r is r % T
    float eps;
};

__device__ __forceinline__ float block_sum_256(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kPrologueThreads / 32; ++i) t += red[i];
    return t;
}

__global__ void __launch_bounds__(kPrologueThreads)
qk_norm_rope_kernel(const PrologueParams p) {
    __shared__ float red_q[8], red_k[8];
    const long long row = blockIdx.x;
    const int t = static_cast<int>(row % p.T);
    const int h = threadIdx.x >> 4;
    const int j = threadIdx.x & 15;
    const int d_lo = h * kHeadDim + 4 * j;  // column of the first element of the pair block
    const int d_hi = d_lo + 64;
    const float* qr = p.q + row * p.ld_in;
    const float* kr = p.k + row * p.ld_in;
    const float* vr = p.v + row * p.ld_in;

    const float4 qa = *reinterpret_cast<const float4*>(qr + d_lo);
    const float4 qb = *reinterpret_cast<const float4*>(qr + d_hi);
    const float4 ka = *reinterpret_cast<const float4*>(kr + d_lo);
    const float4 kb = *reinterpret_cast<const float4*>(kr + d_hi);
    // v: this thread converts 8 consecutive elements
    const float4 va = *reinterpret_cast<const float4*>(vr + 8 * threadIdx.x);
    const float4 vb = *reinterpret_cast<const float4*>(vr + 8 * threadIdx.x + 4);

    float sq = qa.x * qa.x + qa.y * qa.y + qa.z * qa.z + qa.w * qa.w + qb.x * qb.x + qb.y * qb.y + qb.z * qb.z +
               qb.w * qb.w;
    float sk = ka.x * ka.x + ka.y * ka.y + ka.z * ka.z + ka.w * ka.w + kb.x * kb.x + kb.y * kb.y + kb.z * kb.z +
               kb.w * kb.w;
    sq = block_sum_256(sq, red_q);
    sk = block_sum_256(sk, red_k);
    const float rq = sqrtf(sq / (float)kDModel + p.eps);
    const float rk = sqrtf(sk / (float)kDModel + p.eps);

    const float* cs = p.cos_t + (long long)t * kHeadDim + 4 * j;
    const float* sn = p.sin_t + (long long)t * kHeadDim + 4 * j;
    const float4 c_lo = *reinterpret_cast<const float4*>(cs);
    const float4 c_hi = *reinterpret_cast<const float4*>(cs + 64);
    const float4 s_lo = *reinterpret_cast<const float4*>(sn);
    const float4 s_hi = *reinterpret_cast<const float4*>(sn + 64);
    const float4 gq_lo = *reinterpret_cast<const float4*>(p.q_gain + d_lo);
    const float4 gq_hi = *reinterpret_cast<const float4*>(p.q_gain + d_hi);
    const float4 gk_lo = *reinterpret_cast<const float4*>(p.k_gain + d_lo);
    const float4 gk_hi = *reinterpret_cast<const float4*>(p.k_gain + d_hi);

    auto rot = [&](float4 a, float4 b, float r, float4 ga, float4 gb, __nv_bfloat16* out) {
        // normalise (x / rms * g), then rotate-half with this position's tables
        const float a0 = a.x / r * ga.x, a1 = a.y / r * ga.y, a2 = a.z / r * ga.z, a3 = a.w / r * ga.w;
        const float b0 = b.x / r * gb.x, b1 = b.y / r * gb.y, b2 = b.z / r * gb.z, b3 = b.w / r * gb.w;
        uint2 lo, hi;
        lo.x = pack_bf16x2(a0 * c_lo.x - b0 * s_lo.x, a1 * c_lo.y - b1 * s_lo.y);
        lo.y = pack_bf16x2(a2 * c_lo.z - b2 * s_lo.z, a3 * c_lo.w - b3 * s_lo.w);
        hi.x = pack_bf16x2(b0 * c_hi.x + a0 * s_hi.x, b1 * c_hi.y + a1 * s_hi.y);
        hi.y = pack_bf16x2(b2 * c_hi.z + a2 * s_hi.z, b3 * c_hi.w + a3 * s_hi.w);
        *reinterpret_cast<uint2*>(out + row * kDModel + d_lo) = lo;
        *reinterpret_cast<uint2*>(out + row * kDModel + d_hi) = hi;
    };
    rot(qa, qb, rq, gq_lo, gq_hi, p.qo);
    rot(ka, kb, rk, gk_lo, gk_hi, p.ko);

    uint4 vw;
    vw.x = pack_bf16x2(va.x, va.y);
    vw.y = pack_bf16x2(va.z, va.w);
    vw.z = pack_bf16x2(vb.x, vb.y);
    vw.w = pack_bf16x2(vb.z, vb.w);
    *reinterpret_cast<uint4*>(p.vo + row * kDModel + 8 * threadIdx.x) = vw;
}

}  // namespace elem
}  // namespace dt
