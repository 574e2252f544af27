// Attention backward for sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces the reference's flash_attention_backward (FlashAttention.cpp:185-359,
// declared FlashAttention.h:33-43): given dO, O, the forward statistics m
// (row max of the scaled scores) and l (sum of exp(s - m)), and Q, K, V, it
// returns
//   P  = exp(scale * Q K^T - m) / l          (0 where q_pos < k_pos when causal)
//   dP = dO V^T,   D = rowsum(O * dO),   dS = P * (dP - D) * scale
//   dV = P^T dO,   dK = dS^T Q,   dQ = dS K.
// Three kernels:
//   flash_bwd_pre_kernel   D, lse2 = m*log2(e) + log2(l) per row ([B, H, Tpad],
//                          +inf / 0 in the padding rows), and a bf16 copy of dO;
//   flash_bwd_dkdv_kernel  one CTA per (b, h, 128-key block), K and V resident,
//                          looping over the 128-query blocks that see the keys:
//                          S^T = K Q^T and dP^T = V dO^T into TMEM, P^T and dS^T
//                          written back over them as bf16, then dV += P^T dO and
//                          dK += dS^T Q accumulate in TMEM (512 columns);
//   flash_bwd_dq_kernel    one CTA per (b, h, 128-query block), Q and dO resident,
//                          looping over key blocks: S = Q K^T, dP = dO V^T,
//                          dS over dP, dQ += dS K in TMEM.
// Splitting dQ from dK/dV costs two extra products per tile pair (S and dP are
// computed twice) but needs no atomics and keeps each kernel within TMEM.
// Operands are bf16 in the [B, T, H, D] token-major layout read through the
// same 4-D tensor maps as the forward; accumulation and softmax math are fp32.
#pragma once
#include "dt_common.cuh"

namespace dt {
namespace flash_bwd {

constexpr int kD = 128;
constexpr int kBM = 128;  // rows of a Q or K/V block
constexpr int kTileBytes = kBM * kD * 2;   // 32 KB: 128 rows x 128 dims bf16
constexpr int kHalfBytes = kTileBytes / 2; // one 64-dim half (128-byte swizzle span)
// warps 0-7 math: warp w owns TMEM lanes 32*(w%4)..+31 and column half w/4 of
// every row (the backward's elementwise math needs no row reduction, so the two
// halves never talk); warp 8 TMA, warp 9 MMA; warps 10-11 only complete the
// third warpgroup (registers are granted per warpgroup).
constexpr int kThreads = 384;
constexpr int kTmaWarp = 8, kMmaWarp = 9;
constexpr int kKvStages = 4;               // dq kernel: K_j, V_j ring (two key blocks in flight)

// ---------------------------------------------------------------------------
// Preprocessing: D[row] = O[row] . dO[row], lse2[row] = m*log2(e) + log2(l),
// dO -> bf16.  One warp per (b, h, t) row of 128 dims; t runs over Tpad
// (the padding rows get D = 0, lse2 = +inf so that P = 0 there).
// FlashAttention.cpp:232-237 (D), :262-275 (P from the saved m and l).
// ---------------------------------------------------------------------------
struct PreParams {
    const float* out;                 // fp32 O [B,T,H,D], or null when out_bf16 is given
    const __nv_bfloat16* out_bf16;    // bf16 O [B,T,H,D]
    long long out_row_stride;         // elements between tokens of O
    const float* dout;                // fp32 dO [B,T,H,D]
    const float* m;                   // [B,T,H]
    const float* l;                   // [B,T,H]
    __nv_bfloat16* dout_bf16;         // [B,T,H,D]
    float* dvec;                      // [B,H,Tpad]
    float* lse2;                      // [B,H,Tpad]
    int B, T, H, Tpad;
};

__global__ void __launch_bounds__(256) flash_bwd_pre_kernel(const PreParams p) {
    const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const long long nrows = (long long)p.B * p.H * p.Tpad;
    if (row >= nrows) return;
    const int t = (int)(row % p.Tpad);
    const long long bh = row / p.Tpad;
    const int h = (int)(bh % p.H);
    const int b = (int)(bh / p.H);
    float dsum = 0.f, lse = INFINITY;
    if (t < p.T) {
        const long long tok = (long long)b * p.T + t;
        const long long gi = (tok * p.H + h) * kD + lane * 4;
        const float4 d4 = *reinterpret_cast<const float4*>(p.dout + gi);
        float4 o4;
        if (p.out) {
            o4 = *reinterpret_cast<const float4*>(p.out + tok * p.out_row_stride + (long long)h * kD + lane * 4);
        } else {
            const uint2 w = *reinterpret_cast<const uint2*>(p.out_bf16 + tok * p.out_row_stride + (long long)h * kD +
                                                            lane * 4);
            o4.x = __uint_as_float(w.x << 16);
            o4.y = __uint_as_float(w.x & 0xffff0000u);
            o4.z = __uint_as_float(w.y << 16);
            o4.w = __uint_as_float(w.y & 0xffff0000u);
        }
        dsum = o4.x * d4.x + o4.y * d4.y + o4.z * d4.z + o4.w * d4.w;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, off);
        *reinterpret_cast<uint2*>(p.dout_bf16 + gi) = make_uint2(pack_bf16x2(d4.x, d4.y), pack_bf16x2(d4.z, d4.w));
        const long long si = tok * p.H + h;
        const float lv = p.l[si];
        lse = (lv > 0.f) ? p.m[si] * 1.4426950408889634f + __log2f(lv) : INFINITY;
    }
    if (lane == 0) {
        p.dvec[row] = dsum;
        p.lse2[row] = lse;
    }
}

struct Params {
    int B, T, H;
    int nblk;            // ceil(T / 128)
    int Tpad;            // nblk * 128: row stride of dvec / lse2
    int causal;
    float scale;         // caller's scale (reference: 1/sqrt(head_dim))
    float scale_log2;    // scale * log2(e)
    const float* dvec;   // [B,H,Tpad]
    const float* lse2;   // [B,H,Tpad]
    float* dq;           // [B,T,H,D] fp32 (dq kernel)
    float* dk;           // [B,T,H,D] fp32 (dkdv kernel)
    float* dv;           // [B,T,H,D] fp32 (dkdv kernel)
};

enum : unsigned { kSiteLoad = 0x61, kSiteEmpty, kSiteS, kSiteP, kSiteAcc, kSiteDone };

// 1-D bulk copy global -> shared (this CTA), completing on `bar`.  Both addresses
// 16-byte aligned and `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(smem_dst)),
                 "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Stores 32 fp32 values as columns [col0, col0+32) of row (b, t, h) of a [B,T,H,D] array.
__device__ __forceinline__ void store_row_chunk(float* base, const Params& p, int b, int t, int h, int col0,
                                                const float (&v)[32]) {
    float4* d4 = reinterpret_cast<float4*>(base + (((long long)b * p.T + t) * p.H + h) * kD + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

// K-major operand (128 rows x 128 dims in two 64-dim halves), 16-wide K step kk.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t tile, int kk) {
    return umma_desc_sw128(tile + (uint32_t)((kk >> 2) * kHalfBytes + (kk & 3) * 32), 16, 1024);
}
// The same tile read MN-major (N = dims, K = rows), 16 rows per step kk.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t tile, int kk) {
    return umma_desc_sw128(tile + (uint32_t)(kk * 2048), kHalfBytes, 1024);
}

// TMEM column of the packed bf16 pairs for 16-wide step kk of a 128-column
// S/dP tile: column half 0 packs into columns [0, 32), half 1 into [64, 96)
// (each half overwrites only columns it has already read).
__device__ __forceinline__ uint32_t packed_col(int kk) { return (uint32_t)(kk * 8 + (kk >= 4 ? 32 : 0)); }

// ---------------------------------------------------------------------------
// dK, dV: CTA = (b, h, key block kb); query blocks i = (causal ? kb : 0) .. nblk-1.
// ---------------------------------------------------------------------------
struct __align__(1024) SmemKV {
    uint8_t k[kTileBytes];
    uint8_t v[kTileBytes];
    uint8_t q[2][kTileBytes];
    uint8_t dout[2][kTileBytes];
    float lse[2][kBM];
    float dvec[2][kBM];
    uint64_t kv_full;
    uint64_t st_full[2];
    uint64_t st_empty[2];
    uint64_t s_full;
    uint64_t pd_full;
    uint64_t acc_done;
    uint64_t mma_done;
    uint32_t tmem_base;
};

__global__ void __launch_bounds__(kThreads, 1)
flash_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v, const __grid_constant__ CUtensorMap tmap_do,
                      const Params p) {
    extern __shared__ uint8_t smem_raw[];
    SmemKV& sm = *reinterpret_cast<SmemKV*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int BH = p.B * p.H;
    const int kb = static_cast<int>(blockIdx.x) / BH;  // causal: low kb sees the most query blocks -> first
    const int bh = static_cast<int>(blockIdx.x) % BH;
    const int b = bh / p.H;
    const int h = bh % p.H;
    const int i0 = p.causal ? kb : 0;
    const int nq = p.nblk - i0;

    if (threadIdx.x == 0) {
        mbar_init(&sm.kv_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&sm.st_full[s], 1);
            mbar_init(&sm.st_empty[s], 1);
        }
        mbar_init(&sm.s_full, 1);
        mbar_init(&sm.pd_full, 8);
        mbar_init(&sm.acc_done, 1);
        mbar_init(&sm.mma_done, 1);
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(&sm.tmem_base, 512);
        tmem_relinquish();
    }
    if (warp == kTmaWarp && lane == 0) {
        tma_prefetch_desc(&tmap_q);
        tma_prefetch_desc(&tmap_k);
        tma_prefetch_desc(&tmap_v);
        tma_prefetch_desc(&tmap_do);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + 256, tdK = tmem + 384;

    if (warp == kTmaWarp) {
        // ------------------------------ TMA producer ------------------------
        if (lane == 0) {
            mbar_arrive_expect_tx(&sm.kv_full, 2 * kTileBytes);
            for (int hf = 0; hf < 2; ++hf) {
                tma_load_4d(sm.k + hf * kHalfBytes, &tmap_k, &sm.kv_full, hf * 64, h, kb * kBM, b);
                tma_load_4d(sm.v + hf * kHalfBytes, &tmap_v, &sm.kv_full, hf * 64, h, kb * kBM, b);
            }
            int issued = 0;
            for (int it = 0; it < nq; ++it) {
                const int s = it & 1;
                if (!mbar_wait(&sm.st_empty[s], ((it >> 1) & 1) ^ 1, kSiteEmpty)) break;
                const int i = i0 + it;
                mbar_arrive_expect_tx(&sm.st_full[s], 2 * kTileBytes + 2 * kBM * 4);
                for (int hf = 0; hf < 2; ++hf) {
                    tma_load_4d(sm.q[s] + hf * kHalfBytes, &tmap_q, &sm.st_full[s], hf * 64, h, i * kBM, b);
                    tma_load_4d(sm.dout[s] + hf * kHalfBytes, &tmap_do, &sm.st_full[s], hf * 64, h, i * kBM, b);
                }
                const long long row0 = (long long)bh * p.Tpad + (long long)i * kBM;
                bulk_load(sm.lse[s], p.lse2 + row0, kBM * 4, &sm.st_full[s]);
                bulk_load(sm.dvec[s], p.dvec + row0, kBM * 4, &sm.st_full[s]);
                ++issued;
            }
            if (error_raised()) {
                // drain copies in flight before the CTA exits
                mbar_wait(&sm.kv_full, 0, kSiteLoad);
                for (int it = max(0, issued - 2); it < issued; ++it)
                    mbar_wait(&sm.st_full[it & 1], (it >> 1) & 1, kSiteLoad);
            }
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------ MMA issuer --------------------------
        if (lane == 0) {
            constexpr uint32_t idesc_ss = umma_idesc_bf16(kBM, kBM, 0, 0);  // both operands K-major
            constexpr uint32_t idesc_ts = umma_idesc_bf16(kBM, kD, 0, 1);   // A in TMEM, B MN-major
            bool ok = mbar_wait(&sm.kv_full, 0, kSiteLoad);
            const uint32_t ka = smem_u32(sm.k), va = smem_u32(sm.v);
            for (int it = 0; ok && it < nq; ++it) {
                const int s = it & 1;
                if (!mbar_wait(&sm.st_full[s], (it >> 1) & 1, kSiteLoad)) { ok = false; break; }
                tc_fence_after();
                const uint32_t qa = smem_u32(sm.q[s]), da = smem_u32(sm.dout[s]);
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk)  // S^T = K Q^T  [keys x queries]
                    umma_ss(tS, desc_kmajor(ka, kk), desc_kmajor(qa, kk), idesc_ss, kk > 0 ? 1u : 0u);
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk)  // dP^T = V dO^T
                    umma_ss(tdP, desc_kmajor(va, kk), desc_kmajor(da, kk), idesc_ss, kk > 0 ? 1u : 0u);
                umma_commit(&sm.s_full);
                if (!mbar_wait(&sm.pd_full, it & 1, kSiteP)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < kBM / 16; ++kk)  // dV += P^T dO   (16 queries per step)
                    umma_ts(tdV, tS + packed_col(kk), desc_mnmajor(da, kk), idesc_ts, (it > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
                for (int kk = 0; kk < kBM / 16; ++kk)  // dK += dS^T Q
                    umma_ts(tdK, tdP + packed_col(kk), desc_mnmajor(qa, kk), idesc_ts, (it > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&sm.st_empty[s]);
            }
            if (ok) umma_commit(&sm.acc_done);
            umma_commit(&sm.mma_done);
            mbar_wait(&sm.mma_done, 0, kSiteDone);
        }
        __syncwarp();
    } else if (warp < 8) {
        // ------------------------------ math warps --------------------------
        // thread = key row kr (TMEM lane); P^T / dS^T over the 64 queries of
        // this warp's column half, in 32-query chunks.
        const int hf = warp >> 2;
        const int kr = (warp & 3) * 32 + lane;
        const int k_pos = kb * kBM + kr;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const float c = p.scale_log2;
        bool ok = true;
        for (int it = 0; it < nq; ++it) {
            const int s = it & 1;
            const int i = i0 + it;
            if (!mbar_wait(&sm.s_full, it & 1, kSiteS)) { ok = false; break; }
            tc_fence_after();
            const bool diag = p.causal && (i == kb);
#pragma unroll 1
            for (int ch = 0; ch < 2; ++ch) {
                const int cc = hf * 2 + ch;  // 32-query chunk of the 128
                float sv[32], dp[32];
                tmem_ld32(tS + lane_off + cc * 32, sv);
                tmem_ld32(tdP + lane_off + cc * 32, dp);
                tmem_wait_ld();
                const float* lse = sm.lse[s] + cc * 32;
                const float* dvec = sm.dvec[s] + cc * 32;
                uint32_t pp[16], pd[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const float2 l2 = *reinterpret_cast<const float2*>(lse + 2 * e);
                    const float2 d2 = *reinterpret_cast<const float2*>(dvec + 2 * e);
                    float p0 = ex2_approx(sv[2 * e] * c - l2.x);
                    float p1 = ex2_approx(sv[2 * e + 1] * c - l2.y);
                    if (diag) {
                        const int q = i * kBM + cc * 32 + 2 * e;
                        if (q < k_pos) p0 = 0.f;
                        if (q + 1 < k_pos) p1 = 0.f;
                    }
                    const float ds0 = p0 * (dp[2 * e] - d2.x) * p.scale;
                    const float ds1 = p1 * (dp[2 * e + 1] - d2.y) * p.scale;
                    pp[e] = pack_bf16x2(p0, p1);
                    pd[e] = pack_bf16x2(ds0, ds1);
                }
                // P^T / dS^T as bf16 pairs: chunk ch of half hf lands in columns
                // [64 hf + 16 ch, +16) of S^T / dP^T, which this warp has read.
                tmem_st16(tS + lane_off + hf * 64 + ch * 16, pp);
                tmem_st16(tdP + lane_off + hf * 64 + ch * 16, pd);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.pd_full);
        }
        // ---- epilogue: dK, dV rows of this key block -------------------------
        if (ok && nq > 0 && mbar_wait(&sm.acc_done, 0, kSiteAcc)) {
            tc_fence_after();
#pragma unroll 1
            for (int cc = hf * 2; cc < hf * 2 + 2; ++cc) {
                float a[32], bq[32];
                tmem_ld32(tdK + lane_off + cc * 32, a);
                tmem_ld32(tdV + lane_off + cc * 32, bq);
                tmem_wait_ld();
                if (k_pos < p.T) {
                    store_row_chunk(p.dk, p, b, k_pos, h, cc * 32, a);
                    store_row_chunk(p.dv, p, b, k_pos, h, cc * 32, bq);
                }
            }
        } else if (nq == 0 && k_pos < p.T) {
            float z[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) z[e] = 0.f;
            for (int cc = hf * 2; cc < hf * 2 + 2; ++cc) {
                store_row_chunk(p.dk, p, b, k_pos, h, cc * 32, z);
                store_row_chunk(p.dv, p, b, k_pos, h, cc * 32, z);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// dQ: CTA = (b, h, query block qb); key blocks j = 0 .. (causal ? qb : nblk-1).
// ---------------------------------------------------------------------------
struct __align__(1024) SmemQ {
    uint8_t q[kTileBytes];
    uint8_t dout[kTileBytes];
    uint8_t kv[kKvStages][kTileBytes];  // K_0, V_0, K_1, V_1, ...
    uint64_t q_full;
    uint64_t kv_full[kKvStages];
    uint64_t kv_empty[kKvStages];
    uint64_t s_full;
    uint64_t ds_full;
    uint64_t acc_done;
    uint64_t mma_done;
    uint32_t tmem_base;
};

__global__ void __launch_bounds__(kThreads, 1)
flash_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                    const __grid_constant__ CUtensorMap tmap_v, const __grid_constant__ CUtensorMap tmap_do,
                    const Params p) {
    extern __shared__ uint8_t smem_raw[];
    SmemQ& sm = *reinterpret_cast<SmemQ*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int BH = p.B * p.H;
    const int qb = p.nblk - 1 - static_cast<int>(blockIdx.x) / BH;  // causal: high qb sees the most keys -> first
    const int bh = static_cast<int>(blockIdx.x) % BH;
    const int b = bh / p.H;
    const int h = bh % p.H;
    const int nk = p.causal ? qb + 1 : p.nblk;

    if (threadIdx.x == 0) {
        mbar_init(&sm.q_full, 1);
        for (int s = 0; s < kKvStages; ++s) {
            mbar_init(&sm.kv_full[s], 1);
            mbar_init(&sm.kv_empty[s], 1);
        }
        mbar_init(&sm.s_full, 1);
        mbar_init(&sm.ds_full, 8);
        mbar_init(&sm.acc_done, 1);
        mbar_init(&sm.mma_done, 1);
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(&sm.tmem_base, 512);
        tmem_relinquish();
    }
    if (warp == kTmaWarp && lane == 0) {
        tma_prefetch_desc(&tmap_q);
        tma_prefetch_desc(&tmap_k);
        tma_prefetch_desc(&tmap_v);
        tma_prefetch_desc(&tmap_do);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    const uint32_t tS = tmem, tdP = tmem + 128, tdQ = tmem + 256;

    if (warp == kTmaWarp) {
        // ------------------------------ TMA producer ------------------------
        if (lane == 0) {
            mbar_arrive_expect_tx(&sm.q_full, 2 * kTileBytes);
            for (int hf = 0; hf < 2; ++hf) {
                tma_load_4d(sm.q + hf * kHalfBytes, &tmap_q, &sm.q_full, hf * 64, h, qb * kBM, b);
                tma_load_4d(sm.dout + hf * kHalfBytes, &tmap_do, &sm.q_full, hf * 64, h, qb * kBM, b);
            }
            int issued = 0;
            for (int L = 0; L < 2 * nk; ++L) {
                const int s = L % kKvStages;
                if (!mbar_wait(&sm.kv_empty[s], ((L / kKvStages) & 1) ^ 1, kSiteEmpty)) break;
                mbar_arrive_expect_tx(&sm.kv_full[s], kTileBytes);
                const int kt = (L >> 1) * kBM;
                for (int hf = 0; hf < 2; ++hf) {
                    if (L & 1) tma_load_4d(sm.kv[s] + hf * kHalfBytes, &tmap_v, &sm.kv_full[s], hf * 64, h, kt, b);
                    else tma_load_4d(sm.kv[s] + hf * kHalfBytes, &tmap_k, &sm.kv_full[s], hf * 64, h, kt, b);
                }
                ++issued;
            }
            if (error_raised()) {
                mbar_wait(&sm.q_full, 0, kSiteLoad);
                for (int L = max(0, issued - kKvStages); L < issued; ++L)
                    mbar_wait(&sm.kv_full[L % kKvStages], (L / kKvStages) & 1, kSiteLoad);
            }
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------ MMA issuer --------------------------
        if (lane == 0) {
            constexpr uint32_t idesc_ss = umma_idesc_bf16(kBM, kBM, 0, 0);
            constexpr uint32_t idesc_ts = umma_idesc_bf16(kBM, kD, 0, 1);
            auto stage = [](int L) { return L % kKvStages; };
            auto phase = [](int L) { return (uint32_t)((L / kKvStages) & 1); };
            const uint32_t qa = smem_u32(sm.q), da = smem_u32(sm.dout);
            bool ok = mbar_wait(&sm.q_full, 0, kSiteLoad);
            if (ok) ok = mbar_wait(&sm.kv_full[stage(0)], phase(0), kSiteLoad);
            if (ok) ok = mbar_wait(&sm.kv_full[stage(1)], phase(1), kSiteLoad);
            if (ok) {
                tc_fence_after();
                const uint32_t ka = smem_u32(sm.kv[stage(0)]), va = smem_u32(sm.kv[stage(1)]);
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk)
                    umma_ss(tS, desc_kmajor(qa, kk), desc_kmajor(ka, kk), idesc_ss, kk > 0 ? 1u : 0u);
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk)
                    umma_ss(tdP, desc_kmajor(da, kk), desc_kmajor(va, kk), idesc_ss, kk > 0 ? 1u : 0u);
                umma_commit(&sm.s_full);
            }
            for (int j = 0; ok && j < nk; ++j) {
                const int LK = 2 * j, LV = 2 * j + 1, LK1 = 2 * j + 2, LV1 = 2 * j + 3;
                const bool next = (j + 1) < nk;
                if (!mbar_wait(&sm.ds_full, j & 1, kSiteP)) { ok = false; break; }
                if (next) {
                    if (!mbar_wait(&sm.kv_full[stage(LK1)], phase(LK1), kSiteLoad)) { ok = false; break; }
                    if (!mbar_wait(&sm.kv_full[stage(LV1)], phase(LV1), kSiteLoad)) { ok = false; break; }
                }
                tc_fence_after();
                // S(j+1) may overwrite S: the math warps have read S(j) (ds_full)
                if (next) {
                    const uint32_t ka1 = smem_u32(sm.kv[stage(LK1)]);
#pragma unroll
                    for (int kk = 0; kk < kD / 16; ++kk)
                        umma_ss(tS, desc_kmajor(qa, kk), desc_kmajor(ka1, kk), idesc_ss, kk > 0 ? 1u : 0u);
                }
                // dQ += dS K_j  (dS: bf16 pairs over the first 64 columns of dP)
                const uint32_t ka = smem_u32(sm.kv[stage(LK)]);
#pragma unroll
                for (int kk = 0; kk < kBM / 16; ++kk)
                    umma_ts(tdQ, tdP + packed_col(kk), desc_mnmajor(ka, kk), idesc_ts, (j > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&sm.kv_empty[stage(LK)]);
                umma_commit(&sm.kv_empty[stage(LV)]);
                // dP(j+1) after dQ(j) has read dS(j) from the same columns (in-order issue)
                if (next) {
                    const uint32_t va1 = smem_u32(sm.kv[stage(LV1)]);
#pragma unroll
                    for (int kk = 0; kk < kD / 16; ++kk)
                        umma_ss(tdP, desc_kmajor(da, kk), desc_kmajor(va1, kk), idesc_ss, kk > 0 ? 1u : 0u);
                    umma_commit(&sm.s_full);
                }
            }
            if (ok) umma_commit(&sm.acc_done);
            umma_commit(&sm.mma_done);
            mbar_wait(&sm.mma_done, 0, kSiteDone);
        }
        __syncwarp();
    } else if (warp < 8) {
        // ------------------------------ math warps --------------------------
        // thread = query row r; dS over the 64 keys of this warp's column half
        // in 32-key chunks, written over dP.
        const int hf = warp >> 2;
        const int r = (warp & 3) * 32 + lane;
        const int q_pos = qb * kBM + r;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const long long srow = (long long)bh * p.Tpad + q_pos;  // q_pos < Tpad always
        const float lse_r = p.lse2[srow];
        const float d_r = p.dvec[srow];
        const float c = p.scale_log2;
        bool ok = true;
        for (int j = 0; j < nk; ++j) {
            if (!mbar_wait(&sm.s_full, j & 1, kSiteS)) { ok = false; break; }
            tc_fence_after();
            const int k0 = j * kBM;
            const bool masked = (p.causal && j == qb) || (k0 + kBM > p.T);
#pragma unroll 1
            for (int ch = 0; ch < 2; ++ch) {
                const int cc = hf * 2 + ch;  // 32-key chunk of the 128
                float sv[32], dp[32];
                tmem_ld32(tS + lane_off + cc * 32, sv);
                tmem_ld32(tdP + lane_off + cc * 32, dp);
                tmem_wait_ld();
                uint32_t pd[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    float p0 = ex2_approx(sv[2 * e] * c - lse_r);
                    float p1 = ex2_approx(sv[2 * e + 1] * c - lse_r);
                    if (masked) {
                        const int key = k0 + cc * 32 + 2 * e;
                        if ((p.causal && key > q_pos) || key >= p.T) p0 = 0.f;
                        if ((p.causal && key + 1 > q_pos) || key + 1 >= p.T) p1 = 0.f;
                    }
                    pd[e] = pack_bf16x2(p0 * (dp[2 * e] - d_r) * p.scale, p1 * (dp[2 * e + 1] - d_r) * p.scale);
                }
                tmem_st16(tdP + lane_off + hf * 64 + ch * 16, pd);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.ds_full);
        }
        if (ok && nk > 0 && mbar_wait(&sm.acc_done, 0, kSiteAcc)) {
            tc_fence_after();
#pragma unroll 1
            for (int cc = hf * 2; cc < hf * 2 + 2; ++cc) {
                float a[32];
                tmem_ld32(tdQ + lane_off + cc * 32, a);
                tmem_wait_ld();
                if (q_pos < p.T) store_row_chunk(p.dq, p, b, q_pos, h, cc * 32, a);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace flash_bwd
}  // namespace dt
