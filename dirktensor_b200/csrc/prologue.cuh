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
    pdl_enter();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
         i += (long long)gridDim.x * blockDim.x) {
        const float4 v = src[i];
        uint2 w;
        w.x = pack_bf16x2(v.x, v.y);
        w.y = pack_bf16x2(v.z, v.w);
        dst[i] = w;
    }
}

// One system-scope fence, launched on the stream right after a kernel that
// stored into peers' memory: the stream orders that kernel's stores before
// this fence, and the fence makes them visible system-wide before whatever
// follows on the stream (the barrier after which the owners read them).  One
// fence here replaces one per storing thread at the end of the kernel.
__global__ void system_fence_kernel() {
    if (threadIdx.x == 0) __threadfence_system();
}

// Barrier of the in-kernel exchange, on every rank after the kernel that stored
// this rank's output rows into the owners' receive buffers: a system-scope
// fence (the stream has ordered that kernel's stores before this one), then
// thread r publishes `epoch` in rank r's flag array at slot `rank` (a release
// store through the peer mapping) and waits until rank r's epoch has arrived
// in this rank's own array (acquire loads).  The wait gives up after 1 second:
// it records the site in the device error word and returns, so a rank that
// never arrives cannot hang the GPU.  One thread per rank, ranks on different
// GPUs; flags only grow (epochs count steps from 1).
struct BarrierArgs {
    unsigned* flags[8];  // flags[r]: rank r's flag array [8] as mapped in this process
    int ranks;
    int rank;
    unsigned epoch;
};
__global__ void exchange_barrier_kernel(const BarrierArgs a) {
    if (threadIdx.x == 0) __threadfence_system();
    __syncthreads();
    const int r = threadIdx.x;
    if (r >= a.ranks) return;
    const unsigned epoch = a.epoch;
    unsigned* slot = a.flags[r] + a.rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(slot), "r"(epoch) : "memory");
    const unsigned* mine = a.flags[a.rank] + r;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
        if ((int)(v - epoch) >= 0) break;
        if ((it & 63u) == 63u) {
            if (error_raised()) break;
            if (globaltimer_ns() - t0 > kWaitBudgetNs) {
                report_error(kDevTimeoutBase | 0x90u, (unsigned)r);
                break;
            }
        }
        __nanosleep(64);
    }
}

// Three tensors in one launch (raw Q, K, V); blockIdx.y selects the tensor.
struct Cast3 {
    const float4* src[3];
    uint2* dst[3];
};
// Each thread keeps kCastUnroll independent 16-byte loads in flight per iteration
// (one at a time left a short cast latency-bound: 96 MB moved at ~74 % of the copy rate).
constexpr int kCastUnroll = 4;
__global__ void cast3_f32_bf16_kernel(Cast3 a, long long n4) {
    const float4* __restrict__ src = a.src[blockIdx.y];
    uint2* __restrict__ dst = a.dst[blockIdx.y];
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i0 = blockIdx.x * (long long)blockDim.x + threadIdx.x; i0 < n4; i0 += kCastUnroll * stride) {
        float4 v[kCastUnroll];
#pragma unroll
        for (int u = 0; u < kCastUnroll; ++u) {
            const long long i = i0 + u * stride;
            if (i < n4) v[u] = src[i];
        }
#pragma unroll
        for (int u = 0; u < kCastUnroll; ++u) {
            const long long i = i0 + u * stride;
            if (i < n4) dst[i] = make_uint2(pack_bf16x2(v[u].x, v[u].y), pack_bf16x2(v[u].z, v[u].w));
        }
    }
}

constexpr int kDModel = 2048;
constexpr int kHeadDim = 128;
constexpr int kPrologueThreads = 256;

struct PrologueParams {
    const float* q;       // [M, ld_in] rows of the projection output (q part)
    const float* k;
    const float* v;       // null: v is not converted (written in bf16 by the projection)
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
    pdl_enter();
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
    // v: this thread converts 8 consecutive elements (v == null: the producer
    // already wrote v in bf16 and the prologue leaves it alone)
    float4 va = make_float4(0.f, 0.f, 0.f, 0.f), vb = va;
    if (p.v) {
        va = *reinterpret_cast<const float4*>(vr + 8 * threadIdx.x);
        vb = *reinterpret_cast<const float4*>(vr + 8 * threadIdx.x + 4);
    }

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

    if (p.v) {
        uint4 vw;
        vw.x = pack_bf16x2(va.x, va.y);
        vw.y = pack_bf16x2(va.z, va.w);
        vw.z = pack_bf16x2(vb.x, vb.y);
        vw.w = pack_bf16x2(vb.z, vb.w);
        *reinterpret_cast<uint4*>(p.vo + row * kDModel + 8 * threadIdx.x) = vw;
    }
}

// The same prologue as a persistent grid (a few CTAs per SM) striding over the
// tokens: each CTA issues the loads of its next token before it reduces and
// writes the current one, so twice the bytes are in flight per CTA, and the
// two block-wide sums share one barrier per token (double-buffered slots).
#ifndef DT_PROLOGUE_PERSISTENT
#define DT_PROLOGUE_PERSISTENT 2
#endif
__global__ void __launch_bounds__(kPrologueThreads, DT_PROLOGUE_PERSISTENT > 0 ? DT_PROLOGUE_PERSISTENT : 1)
qk_norm_rope_loop_kernel(const PrologueParams p, long long M) {
    pdl_enter();
    __shared__ float red[2][2][kPrologueThreads / 32];  // [slot][q, k][warp]
    const int h = threadIdx.x >> 4;
    const int j = threadIdx.x & 15;
    const int w = threadIdx.x >> 5;
    const int d_lo = h * kHeadDim + 4 * j;
    const int d_hi = d_lo + 64;
    const float4 gq_lo = *reinterpret_cast<const float4*>(p.q_gain + d_lo);
    const float4 gq_hi = *reinterpret_cast<const float4*>(p.q_gain + d_hi);
    const float4 gk_lo = *reinterpret_cast<const float4*>(p.k_gain + d_lo);
    const float4 gk_hi = *reinterpret_cast<const float4*>(p.k_gain + d_hi);
    long long row = blockIdx.x;
    if (row >= M) return;
    float4 cur[6], nxt[6];
    auto load = [&](long long r, float4 (&x)[6]) {
        const float* qr = p.q + r * p.ld_in;
        const float* kr = p.k + r * p.ld_in;
        const float* vr = p.v + r * p.ld_in;
        x[0] = *reinterpret_cast<const float4*>(qr + d_lo);
        x[1] = *reinterpret_cast<const float4*>(qr + d_hi);
        x[2] = *reinterpret_cast<const float4*>(kr + d_lo);
        x[3] = *reinterpret_cast<const float4*>(kr + d_hi);
        if (p.v) {
            x[4] = *reinterpret_cast<const float4*>(vr + 8 * threadIdx.x);
            x[5] = *reinterpret_cast<const float4*>(vr + 8 * threadIdx.x + 4);
        }
    };
    auto sq4 = [](float4 a) { return a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w; };
    load(row, cur);
    for (int slot = 0;; slot ^= 1) {
        const long long next = row + gridDim.x;
        if (next < M) load(next, nxt);
        float sq = sq4(cur[0]) + sq4(cur[1]);
        float sk = sq4(cur[2]) + sq4(cur[3]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            sq += __shfl_xor_sync(0xffffffffu, sq, o);
            sk += __shfl_xor_sync(0xffffffffu, sk, o);
        }
        if ((threadIdx.x & 31) == 0) {
            red[slot][0][w] = sq;
            red[slot][1][w] = sk;
        }
        __syncthreads();
        sq = 0.f;
        sk = 0.f;
#pragma unroll
        for (int i = 0; i < kPrologueThreads / 32; ++i) {
            sq += red[slot][0][i];
            sk += red[slot][1][i];
        }
        const float rq = sqrtf(sq / (float)kDModel + p.eps);
        const float rk = sqrtf(sk / (float)kDModel + p.eps);
        const int t = static_cast<int>(row % p.T);
        const float* cs = p.cos_t + (long long)t * kHeadDim + 4 * j;
        const float* sn = p.sin_t + (long long)t * kHeadDim + 4 * j;
        const float4 c_lo = *reinterpret_cast<const float4*>(cs);
        const float4 c_hi = *reinterpret_cast<const float4*>(cs + 64);
        const float4 s_lo = *reinterpret_cast<const float4*>(sn);
        const float4 s_hi = *reinterpret_cast<const float4*>(sn + 64);
        auto rot = [&](float4 a, float4 b, float r, float4 ga, float4 gb, __nv_bfloat16* out) {
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
        rot(cur[0], cur[1], rq, gq_lo, gq_hi, p.qo);
        rot(cur[2], cur[3], rk, gk_lo, gk_hi, p.ko);
        if (p.v)
            *reinterpret_cast<uint4*>(p.vo + row * kDModel + 8 * threadIdx.x) =
                make_uint4(pack_bf16x2(cur[4].x, cur[4].y), pack_bf16x2(cur[4].z, cur[4].w),
                           pack_bf16x2(cur[5].x, cur[5].y), pack_bf16x2(cur[5].z, cur[5].w));
        if (next >= M) break;
        row = next;
#pragma unroll
        for (int i = 0; i < 6; ++i) cur[i] = nxt[i];
    }
}

// ---------------------------------------------------------------------------
// Head-sharded prologue (heads split over ranks, column-parallel QKV).  The
// QK-RMSNorm sums squares over all 2048 columns of a token, i.e. over every
// rank's heads (RMSNorm.cpp:17, applied at OlmoAttention.cpp:70,76), so it runs
// in two steps around one all-reduce of 2 floats per token:
//   qk_sumsq_kernel            ss[row] = {sum q^2, sum k^2} over this rank's
//                              `width` = heads * 128 columns;
//   (all-reduce ss over the ranks: the full-row sums)
//   qk_norm_rope_shard_kernel  y = x / sqrt(ss / 2048 + eps) * g, RoPE, bf16,
//                              for this rank's heads only.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
qk_sumsq_kernel(const float* __restrict__ q, const float* __restrict__ k, long long ld, int width, long long M,
                float2* __restrict__ ss) {
    // one warp per token
    const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= M) return;
    const float4* qr = reinterpret_cast<const float4*>(q + row * ld);
    const float4* kr = reinterpret_cast<const float4*>(k + row * ld);
    float sq = 0.f, sk = 0.f;
    for (int c = lane; c < width / 4; c += 32) {
        const float4 a = qr[c], b = kr[c];
        sq += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
        sk += b.x * b.x + b.y * b.y + b.z * b.z + b.w * b.w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
    }
    if (lane == 0) ss[row] = make_float2(sq, sk);
}

struct ShardPrologueParams {
    const float* q;       // [M, ld_in]: this rank's q columns (width = heads * 128)
    const float* k;
    const float* v;
    long long ld_in;
    const float2* ss;     // [M] full-row sums of squares {q, k}
    const float* q_gain;  // [width]: this rank's slice of the 2048 gains
    const float* k_gain;
    const float* sin_t;   // [max_seq, 128]
    const float* cos_t;
    __nv_bfloat16* qo;    // [M, width]
    __nv_bfloat16* ko;
    __nv_bfloat16* vo;
    int heads;            // 1, 2, 4, 8 or 16
    int T;
    long long M;
    float eps;
};

// 16 threads per (token, head), as qk_norm_rope_kernel; a CTA of 256 threads
// covers 16 / heads tokens.
__global__ void __launch_bounds__(kPrologueThreads)
qk_norm_rope_shard_kernel(const ShardPrologueParams p) {
    const int per_tok = p.heads * 16;
    const long long row = (long long)blockIdx.x * (kPrologueThreads / per_tok) + threadIdx.x / per_tok;
    if (row >= p.M) return;
    const int tid = threadIdx.x % per_tok;
    const int h = tid >> 4;
    const int j = tid & 15;
    const int width = p.heads * kHeadDim;
    const int t = static_cast<int>(row % p.T);
    const int d_lo = h * kHeadDim + 4 * j;
    const int d_hi = d_lo + 64;
    const float* qr = p.q + row * p.ld_in;
    const float* kr = p.k + row * p.ld_in;
    const float* vr = p.v + row * p.ld_in;
    const float4 qa = *reinterpret_cast<const float4*>(qr + d_lo);
    const float4 qb = *reinterpret_cast<const float4*>(qr + d_hi);
    const float4 ka = *reinterpret_cast<const float4*>(kr + d_lo);
    const float4 kb = *reinterpret_cast<const float4*>(kr + d_hi);
    const float4 va = *reinterpret_cast<const float4*>(vr + 8 * tid);
    const float4 vb = *reinterpret_cast<const float4*>(vr + 8 * tid + 4);
    const float2 s2 = p.ss[row];
    const float rq = sqrtf(s2.x / (float)kDModel + p.eps);
    const float rk = sqrtf(s2.y / (float)kDModel + p.eps);
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
        const float a0 = a.x / r * ga.x, a1 = a.y / r * ga.y, a2 = a.z / r * ga.z, a3 = a.w / r * ga.w;
        const float b0 = b.x / r * gb.x, b1 = b.y / r * gb.y, b2 = b.z / r * gb.z, b3 = b.w / r * gb.w;
        uint2 lo, hi;
        lo.x = pack_bf16x2(a0 * c_lo.x - b0 * s_lo.x, a1 * c_lo.y - b1 * s_lo.y);
        lo.y = pack_bf16x2(a2 * c_lo.z - b2 * s_lo.z, a3 * c_lo.w - b3 * s_lo.w);
        hi.x = pack_bf16x2(b0 * c_hi.x + a0 * s_hi.x, b1 * c_hi.y + a1 * s_hi.y);
        hi.y = pack_bf16x2(b2 * c_hi.z + a2 * s_hi.z, b3 * c_hi.w + a3 * s_hi.w);
        *reinterpret_cast<uint2*>(out + row * width + d_lo) = lo;
        *reinterpret_cast<uint2*>(out + row * width + d_hi) = hi;
    };
    rot(qa, qb, rq, gq_lo, gq_hi, p.qo);
    rot(ka, kb, rk, gk_lo, gk_hi, p.ko);
    *reinterpret_cast<uint4*>(p.vo + row * width + 8 * tid) =
        make_uint4(pack_bf16x2(va.x, va.y), pack_bf16x2(va.z, va.w), pack_bf16x2(vb.x, vb.y), pack_bf16x2(vb.z, vb.w));
}

}  // namespace elem
}  // namespace dt

namespace dt {
namespace elem {

// ---------------------------------------------------------------------------
// Backward of QK-RMSNorm + RoPE (OlmoAttention.cpp:149-187 and :228-237,
// RMSNorm.cpp:24-36), fused per token, plus the bf16 packing of dV:
//   dn = RoPE^T(dq_rope)            d_in[d] = dy[d] c[d] + dy[d+64] s[d+64],
//                                    d_in[d+64] = -dy[d] s[d] + dy[d+64] c[d+64]
//   rms = sqrt(mean(x^2) + eps),  x_hat = x / rms,  y = x_hat * g
//   c = mean(dn * y),  dx = (g * dn - x_hat * c) / rms,  dg += dn * x_hat
// (x = the projection before the norm, which the forward left in its fp32
// [q|k|v] buffer).  Writes dx of q and k and the bf16 dV into one
// [M, 3*2048] bf16 row (the operand of the projection-gradient GEMMs).  A CTA
// of 256 threads walks kBwdRows tokens with the forward's thread layout (thread
// = 4 RoPE pairs of one head), keeping its gain-gradient partial sums in
// registers and writing them to gain_part[blockIdx.x] (q gains, then k gains);
// gain_grad_reduce_kernel then adds the partials in CTA order into dqg / dkg,
// so the result does not depend on scheduling (no atomics).
// ---------------------------------------------------------------------------
constexpr int kBwdRows = 32;

struct NormRopeBwdParams {
    const float* dq;      // [M, 2048] gradient of the RoPE'd q
    const float* dk;      // [M, 2048]
    const float* dv;      // [M, 2048]
    const float* xq;      // pre-norm q, row stride ld_x
    const float* xk;      // pre-norm k
    long long ld_x;
    const float* q_gain;
    const float* k_gain;
    const float* sin_t;
    const float* cos_t;
    __nv_bfloat16* dqkv;  // [M, 3*2048]
    float* gain_part;     // [gridDim.x, 2 * 2048] per-CTA partial gain gradients
    long long M;
    int T;
    float eps;
};

__global__ void __launch_bounds__(kPrologueThreads)
qk_norm_rope_bwd_kernel(const NormRopeBwdParams p) {
    __shared__ float red[4][kPrologueThreads / 32];
    const int h = threadIdx.x >> 4;
    const int j = threadIdx.x & 15;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int d_lo = h * kHeadDim + 4 * j;
    const int d_hi = d_lo + 64;
    const float4 gq_lo = *reinterpret_cast<const float4*>(p.q_gain + d_lo);
    const float4 gq_hi = *reinterpret_cast<const float4*>(p.q_gain + d_hi);
    const float4 gk_lo = *reinterpret_cast<const float4*>(p.k_gain + d_lo);
    const float4 gk_hi = *reinterpret_cast<const float4*>(p.k_gain + d_hi);
    float accq[8], acck[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) accq[i] = acck[i] = 0.f;
    const long long r0 = (long long)blockIdx.x * kBwdRows;
    for (int rr = 0; rr < kBwdRows; ++rr) {
        const long long row = r0 + rr;
        if (row >= p.M) break;  // uniform across the CTA
        const int t = static_cast<int>(row % p.T);
        const float4 c_lo = *reinterpret_cast<const float4*>(p.cos_t + (long long)t * kHeadDim + 4 * j);
        const float4 c_hi = *reinterpret_cast<const float4*>(p.cos_t + (long long)t * kHeadDim + 4 * j + 64);
        const float4 s_lo = *reinterpret_cast<const float4*>(p.sin_t + (long long)t * kHeadDim + 4 * j);
        const float4 s_hi = *reinterpret_cast<const float4*>(p.sin_t + (long long)t * kHeadDim + 4 * j + 64);
        float dn[2][8], xv[2][8];
        const float* dsrc[2] = {p.dq + row * kDModel, p.dk + row * kDModel};
        const float* xsrc[2] = {p.xq + row * p.ld_x, p.xk + row * p.ld_x};
        float part[4] = {0.f, 0.f, 0.f, 0.f};  // sum x^2 (q, k), sum dn*x*g (q, k)
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const float4 ylo = *reinterpret_cast<const float4*>(dsrc[u] + d_lo);
            const float4 yhi = *reinterpret_cast<const float4*>(dsrc[u] + d_hi);
            const float4 xlo = *reinterpret_cast<const float4*>(xsrc[u] + d_lo);
            const float4 xhi = *reinterpret_cast<const float4*>(xsrc[u] + d_hi);
            const float yl[4] = {ylo.x, ylo.y, ylo.z, ylo.w}, yh[4] = {yhi.x, yhi.y, yhi.z, yhi.w};
            const float cl[4] = {c_lo.x, c_lo.y, c_lo.z, c_lo.w}, ch[4] = {c_hi.x, c_hi.y, c_hi.z, c_hi.w};
            const float sl[4] = {s_lo.x, s_lo.y, s_lo.z, s_lo.w}, sh[4] = {s_hi.x, s_hi.y, s_hi.z, s_hi.w};
            const float4 glo = u ? gk_lo : gq_lo, ghi = u ? gk_hi : gq_hi;
            const float gl[4] = {glo.x, glo.y, glo.z, glo.w}, gh[4] = {ghi.x, ghi.y, ghi.z, ghi.w};
            xv[u][0] = xlo.x; xv[u][1] = xlo.y; xv[u][2] = xlo.z; xv[u][3] = xlo.w;
            xv[u][4] = xhi.x; xv[u][5] = xhi.y; xv[u][6] = xhi.z; xv[u][7] = xhi.w;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                dn[u][e] = yl[e] * cl[e] + yh[e] * sh[e];
                dn[u][4 + e] = -yl[e] * sl[e] + yh[e] * ch[e];
                part[u] += xv[u][e] * xv[u][e] + xv[u][4 + e] * xv[u][4 + e];
                part[2 + u] += dn[u][e] * xv[u][e] * gl[e] + dn[u][4 + e] * xv[u][4 + e] * gh[e];
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) part[k] += __shfl_xor_sync(0xffffffffu, part[k], o);
            if (lane == 0) red[k][wid] = part[k];
        }
        __syncthreads();
        float tot[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < kPrologueThreads / 32; ++w) s += red[k][w];
            tot[k] = s;
        }
        __syncthreads();  // `red` is rewritten by the next row
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const float rms = sqrtf(tot[u] / (float)kDModel + p.eps);
            const float c = tot[2 + u] / rms / (float)kDModel;  // mean(dn * y), y = x / rms * g
            const float4 glo = u ? gk_lo : gq_lo, ghi = u ? gk_hi : gq_hi;
            const float g8[8] = {glo.x, glo.y, glo.z, glo.w, ghi.x, ghi.y, ghi.z, ghi.w};
            float dx[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float xh = xv[u][e] / rms;
                dx[e] = (g8[e] * dn[u][e] - xh * c) / rms;
                if (u) acck[e] += dn[u][e] * xh;
                else accq[e] += dn[u][e] * xh;
            }
            __nv_bfloat16* out = p.dqkv + row * (3 * kDModel) + u * kDModel;
            *reinterpret_cast<uint2*>(out + d_lo) = make_uint2(pack_bf16x2(dx[0], dx[1]), pack_bf16x2(dx[2], dx[3]));
            *reinterpret_cast<uint2*>(out + d_hi) = make_uint2(pack_bf16x2(dx[4], dx[5]), pack_bf16x2(dx[6], dx[7]));
        }
        // dV: 8 consecutive elements per thread
        const float4 va = *reinterpret_cast<const float4*>(p.dv + row * kDModel + 8 * threadIdx.x);
        const float4 vb = *reinterpret_cast<const float4*>(p.dv + row * kDModel + 8 * threadIdx.x + 4);
        *reinterpret_cast<uint4*>(p.dqkv + row * (3 * kDModel) + 2 * kDModel + 8 * threadIdx.x) =
            make_uint4(pack_bf16x2(va.x, va.y), pack_bf16x2(va.z, va.w), pack_bf16x2(vb.x, vb.y),
                       pack_bf16x2(vb.z, vb.w));
    }
    float* part = p.gain_part + (long long)blockIdx.x * (2 * kDModel);
    *reinterpret_cast<float4*>(part + d_lo) = make_float4(accq[0], accq[1], accq[2], accq[3]);
    *reinterpret_cast<float4*>(part + d_hi) = make_float4(accq[4], accq[5], accq[6], accq[7]);
    *reinterpret_cast<float4*>(part + kDModel + d_lo) = make_float4(acck[0], acck[1], acck[2], acck[3]);
    *reinterpret_cast<float4*>(part + kDModel + d_hi) = make_float4(acck[4], acck[5], acck[6], acck[7]);
}

// Adds the per-CTA partial gain gradients [nparts, 2*2048] in order into
// dqg [2048] and dkg [2048] (one thread per column).
__global__ void gain_grad_reduce_kernel(const float* __restrict__ part, int nparts, float* __restrict__ dqg,
                                        float* __restrict__ dkg) {
    const int col = blockIdx.x * blockDim.x + threadIdx.x;
    if (col >= 2 * kDModel) return;
    float acc = 0.f;
    for (int i = 0; i < nparts; ++i) acc += part[(long long)i * (2 * kDModel) + col];
    if (col < kDModel) dqg[col] += acc;
    else dkg[col - kDModel] += acc;
}

// SGD step (OlmoAttention.cpp:315-322, RMSNorm.cpp:38-41): w -= lr * g on the
// fp32 master weights, and optionally refresh their bf16 working copy.
__global__ void sgd_kernel(float* __restrict__ w, const float* __restrict__ g, __nv_bfloat16* __restrict__ wb,
                           float lr, long long n) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float v = w[i] - lr * g[i];
        w[i] = v;
        if (wb) wb[i] = __float2bfloat16_rn(v);
    }
}

}  // namespace elem
}  // namespace dt
