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
//   attn_bwd_pre_kernel   D, lse2 = m*log2(e) + log2(l) per row ([B, H, Tpad],
//                          +inf / 0 in the padding rows), and a bf16 copy of dO;
//   attn_bwd_dkdv_kernel  one CTA per (b, h, 128-key block), K and V resident,
//                          looping over the 128-query blocks that see the keys:
//                          S^T = K Q^T and dP^T = V dO^T into TMEM, P^T and dS^T
//                          written back over them as bf16, then dV += P^T dO and
//                          dK += dS^T Q accumulate in TMEM (512 columns);
//   attn_bwd_dq_kernel    one CTA per (b, h, 128-query block), Q and dO resident,
//                          looping over key blocks: S = Q K^T, dP = dO V^T,
//                          dS over dP, dQ += dS K in TMEM.
// Splitting dQ from dK/dV costs two extra products per tile pair (S and dP are
// computed twice) but needs no atomics and keeps each kernel within TMEM.
// Operands are bf16 in the [B, T, H, D] token-major layout read through the
// same 4-D tensor maps as the forward; accumulation and softmax math are fp32.
#pragma once
#include "dt_common.cuh"

namespace dt {
namespace attn_bwd {

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

__global__ void __launch_bounds__(256) attn_bwd_pre_kernel(const PreParams p) {
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

// Coalesced form of store_row_chunk for a warp: lane i holds row t0 + i.  The 32 x 32
// block passes through `stage` (4 KB of shared memory owned by this warp; 16-byte chunk
// j of row r at position j ^ (r & 7), so writes and reads use every bank), then each
// store instruction writes four whole 128-byte row segments.  Rows t >= T are skipped.
__device__ __forceinline__ void store_rows_staged(float* base, const Params& p, int b, int t0, int h, int col0,
                                                  const float (&v)[32], uint32_t stage, int lane) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(stage + (uint32_t)lane * 128 +
                                                                      ((uint32_t)(j ^ (lane & 7)) << 4)),
                     "f"(v[4 * j]), "f"(v[4 * j + 1]), "f"(v[4 * j + 2]), "f"(v[4 * j + 3])
                     : "memory");
    __syncwarp();
    const int j = lane & 7;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = 4 * i + (lane >> 3);
        float4 x;
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(x.x), "=f"(x.y), "=f"(x.z), "=f"(x.w)
                     : "r"(stage + (uint32_t)r * 128 + ((uint32_t)(j ^ (r & 7)) << 4)));
        const int t = t0 + r;
        if (t < p.T)
            *reinterpret_cast<float4*>(base + (((long long)b * p.T + t) * p.H + h) * kD + col0 + 4 * j) = x;
    }
    __syncwarp();  // the next block reuses the stage
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
//
// TMEM holds S^T, dP^T and the dV, dK accumulators (4 x 128 columns), so S^T and
// dP^T have one buffer each.  The math warps load S^T_i, release its columns at
// once (s_free) and keep P_i in registers; after dP^T_i lands they compute dS_i
// and write P_i and dS_i, both as bf16 pairs, into the dP^T columns they have
// read (per column half: dS into the first 32, P into the next 32).  So the MMA
// thread issues S^T_{i+1} = K Q_{i+1}^T while P_i is still being computed, and
// per query block:
//   [S^T_i read]      S^T_{i+1}
//   [P_i, dS_i ready] dV += P_i^T dO_i, dK += dS_i^T Q_i, dP^T_{i+1} = V dO_{i+1}^T
//                     (the last over P_i / dS_i, in order).
// Q_i (with its lse2 and D rows) and dO_i sit in separate two-stage rings: dO_i
// is free after dV_i, Q_i after dK_i.
// ---------------------------------------------------------------------------
struct __align__(1024) SmemKV {
    uint8_t k[kTileBytes];
    uint8_t v[kTileBytes];
    uint8_t q[2][kTileBytes];
    uint8_t dout[2][kTileBytes];
    float lse[2][kBM];   // travels with q[s]
    float dvec[2][kBM];  // travels with q[s]: the dS phase reads it after dV_i may have freed dout[s]
    uint64_t kv_full;
    uint64_t q_full[2];
    uint64_t q_empty[2];
    uint64_t do_full[2];
    uint64_t do_empty[2];
    uint64_t s_full;
    uint64_t s_free;
    uint64_t dp_full;
    uint64_t pds_full;
    uint64_t acc_done;
    uint64_t mma_done;
    uint32_t tmem_base;
};

__global__ void __launch_bounds__(kThreads, 1)
attn_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
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
            mbar_init(&sm.q_full[s], 1);
            mbar_init(&sm.q_empty[s], 1);
            mbar_init(&sm.do_full[s], 1);
            mbar_init(&sm.do_empty[s], 1);
        }
        mbar_init(&sm.s_full, 1);
        mbar_init(&sm.s_free, 8);
        mbar_init(&sm.dp_full, 1);
        mbar_init(&sm.pds_full, 8);
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
            int issued_q = 0, issued_do = 0;
            for (int it = 0; it < nq; ++it) {
                const int s = it & 1;
                const uint32_t empty_phase = ((it >> 1) & 1) ^ 1;
                const int i = i0 + it;
                if (!mbar_wait(&sm.q_empty[s], empty_phase, kSiteEmpty)) break;
                mbar_arrive_expect_tx(&sm.q_full[s], kTileBytes + 2 * kBM * 4);
                for (int hf = 0; hf < 2; ++hf)
                    tma_load_4d(sm.q[s] + hf * kHalfBytes, &tmap_q, &sm.q_full[s], hf * 64, h, i * kBM, b);
                const long long row0 = (long long)bh * p.Tpad + (long long)i * kBM;
                bulk_load(sm.lse[s], p.lse2 + row0, kBM * 4, &sm.q_full[s]);
                bulk_load(sm.dvec[s], p.dvec + row0, kBM * 4, &sm.q_full[s]);
                ++issued_q;
                if (!mbar_wait(&sm.do_empty[s], empty_phase, kSiteEmpty)) break;
                mbar_arrive_expect_tx(&sm.do_full[s], kTileBytes);
                for (int hf = 0; hf < 2; ++hf)
                    tma_load_4d(sm.dout[s] + hf * kHalfBytes, &tmap_do, &sm.do_full[s], hf * 64, h, i * kBM, b);
                ++issued_do;
            }
            if (error_raised()) {
                // drain copies in flight before the CTA exits
                mbar_wait(&sm.kv_full, 0, kSiteLoad);
                for (int it = max(0, issued_q - 2); it < issued_q; ++it)
                    mbar_wait(&sm.q_full[it & 1], (it >> 1) & 1, kSiteLoad);
                for (int it = max(0, issued_do - 2); it < issued_do; ++it)
                    mbar_wait(&sm.do_full[it & 1], (it >> 1) & 1, kSiteLoad);
            }
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------ MMA issuer --------------------------
        if (lane == 0) {
            constexpr uint32_t idesc_ss = umma_idesc_bf16(kBM, kBM, 0, 0);  // both operands K-major
            constexpr uint32_t idesc_ts = umma_idesc_bf16(kBM, kD, 0, 1);   // A in TMEM, B MN-major
            const uint32_t ka = smem_u32(sm.k), va = smem_u32(sm.v);
            bool ok = mbar_wait(&sm.kv_full, 0, kSiteLoad);  // also drains the K/V copies when nq == 0
            if (ok && nq > 0) ok = mbar_wait(&sm.q_full[0], 0, kSiteLoad);
            if (ok && nq > 0) {
                tc_fence_after();
                const uint32_t qa = smem_u32(sm.q[0]);
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk)  // S^T_0 = K Q_0^T  [keys x queries]
                    umma_ss(tS, desc_kmajor(ka, kk), desc_kmajor(qa, kk), idesc_ss, kk > 0 ? 1u : 0u);
                umma_commit(&sm.s_full);
                ok = mbar_wait(&sm.do_full[0], 0, kSiteLoad);
            }
            if (ok) {
                tc_fence_after();
                const uint32_t da = smem_u32(sm.dout[0]);
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk)  // dP^T_0 = V dO_0^T
                    umma_ss(tdP, desc_kmajor(va, kk), desc_kmajor(da, kk), idesc_ss, kk > 0 ? 1u : 0u);
                umma_commit(&sm.dp_full);
            }
            for (int it = 0; ok && it < nq; ++it) {
                const int s = it & 1, s1 = s ^ 1;
                const bool next = it + 1 < nq;
                const uint32_t full_phase1 = ((it + 1) >> 1) & 1;
                const uint32_t qa = smem_u32(sm.q[s]), da = smem_u32(sm.dout[s]);
                if (next) {
                    // S^T_{i+1} as soon as the math warps have read S^T_i
                    if (!mbar_wait(&sm.s_free, it & 1, kSiteP)) { ok = false; break; }
                    if (!mbar_wait(&sm.q_full[s1], full_phase1, kSiteLoad)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t qa1 = smem_u32(sm.q[s1]);
#pragma unroll
                    for (int kk = 0; kk < kD / 16; ++kk)
                        umma_ss(tS, desc_kmajor(ka, kk), desc_kmajor(qa1, kk), idesc_ss, kk > 0 ? 1u : 0u);
                    umma_commit(&sm.s_full);
                }
                if (!mbar_wait(&sm.pds_full, it & 1, kSiteP)) { ok = false; break; }
                tc_fence_after();
                // dK first: its completion frees the Q stage that Q_{i+2} loads into,
                // and that load is on the way to S^T_{i+2}
#pragma unroll
                for (int kk = 0; kk < kBM / 16; ++kk)  // dK += dS^T Q
                    umma_ts(tdK, tdP + packed_col(kk), desc_mnmajor(qa, kk), idesc_ts, (it > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&sm.q_empty[s]);
#pragma unroll
                for (int kk = 0; kk < kBM / 16; ++kk)  // dV += P^T dO   (16 queries per step)
                    umma_ts(tdV, tdP + 32 + packed_col(kk), desc_mnmajor(da, kk), idesc_ts,
                            (it > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&sm.do_empty[s]);
                if (next) {
                    // dP^T_{i+1} over P_i / dS_i: issued after dV and dK, which read them, in order
                    if (!mbar_wait(&sm.do_full[s1], full_phase1, kSiteLoad)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t da1 = smem_u32(sm.dout[s1]);
#pragma unroll
                    for (int kk = 0; kk < kD / 16; ++kk)
                        umma_ss(tdP, desc_kmajor(va, kk), desc_kmajor(da1, kk), idesc_ss, kk > 0 ? 1u : 0u);
                    umma_commit(&sm.dp_full);
                }
            }
            if (ok && nq > 0) umma_commit(&sm.acc_done);
            umma_commit(&sm.mma_done);
            mbar_wait(&sm.mma_done, 0, kSiteDone);
        }
        __syncwarp();
    } else if (warp < 8) {
        // ------------------------------ math warps --------------------------
        // thread = key row kr (TMEM lane); P^T / dS^T over the 64 queries of
        // this warp's column half, in two 32-query chunks (unrolled, so that P
        // stays in registers from the P phase to the dS phase).
        const int hf = warp >> 2;
        const int kr = (warp & 3) * 32 + lane;
        const int k_pos = kb * kBM + kr;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const float c = p.scale_log2;
        bool ok = true;
        for (int it = 0; it < nq; ++it) {
            const int s = it & 1;
            const int i = i0 + it;
            float pr[2][32];
            // warp-uniform waits: each phase synchronises the warp
            if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full, it & 1, kSiteS))) { ok = false; break; }
            tc_fence_after();
            const bool diag = p.causal && (i == kb);
            // both 32-column loads in flight before the one wait; then S^T's
            // columns are free for the next block's product
            tmem_ld32(tS + lane_off + hf * 64, pr[0]);
            tmem_ld32(tS + lane_off + hf * 64 + 32, pr[1]);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.s_free);
#pragma unroll
            for (int ch = 0; ch < 2; ++ch) {
                const float* lse = sm.lse[s] + (hf * 2 + ch) * 32;
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    const float2 l2 = *reinterpret_cast<const float2*>(lse + e);
                    pr[ch][e] = ex2_approx(pr[ch][e] * c - l2.x);
                    pr[ch][e + 1] = ex2_approx(pr[ch][e + 1] * c - l2.y);
                }
            }
            // The causal mask is a separate pass on the diagonal block only:
            // written inside the loop above, its per-element tests cost more
            // than the exponentials on every block.
            if (diag) {
                const int rel = k_pos - i * kBM - hf * 64;  // queries q < k_pos are masked
#pragma unroll
                for (int ch = 0; ch < 2; ++ch)
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        if (ch * 32 + e < rel) pr[ch][e] = 0.f;
            }
            if (!__all_sync(0xffffffffu, mbar_wait(&sm.dp_full, it & 1, kSiteS))) { ok = false; break; }
            tc_fence_after();
            // dP^T one 32-column chunk at a time (with both chunks and P live at
            // once the math warps ran out of registers and spilled).  Chunk ch of
            // half hf: dS^T goes to columns [64 hf + 16 ch, +16) and P^T to
            // [64 hf + 32 + 16 ch, +16) of dP^T.  P^T of chunk 0 lands in chunk 1's
            // columns, so it is stored only after chunk 1 has been loaded.
            uint32_t pp0[16];
#pragma unroll
            for (int ch = 0; ch < 2; ++ch) {
                float dp[32];
                tmem_ld32(tdP + lane_off + hf * 64 + ch * 32, dp);
                tmem_wait_ld();
                if (ch == 1) tmem_st16(tdP + lane_off + hf * 64 + 32, pp0);
                const float* dvec = sm.dvec[s] + (hf * 2 + ch) * 32;
                uint32_t pd[16], pp[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const float2 d2 = *reinterpret_cast<const float2*>(dvec + 2 * e);
                    pd[e] = pack_bf16x2(pr[ch][2 * e] * (dp[2 * e] - d2.x) * p.scale,
                                        pr[ch][2 * e + 1] * (dp[2 * e + 1] - d2.y) * p.scale);
                    pp[e] = pack_bf16x2(pr[ch][2 * e], pr[ch][2 * e + 1]);
                }
                tmem_st16(tdP + lane_off + hf * 64 + ch * 16, pd);
                if (ch == 0) {
#pragma unroll
                    for (int e = 0; e < 16; ++e) pp0[e] = pp[e];
                } else {
                    tmem_st16(tdP + lane_off + hf * 64 + 48, pp);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.pds_full);
        }
        // ---- epilogue: dK, dV rows of this key block -------------------------
        bool got = ok && nq > 0 && mbar_wait(&sm.acc_done, 0, kSiteAcc);
        got = __all_sync(0xffffffffu, got);  // the staged stores synchronise the warp
        if (got) {
            tc_fence_after();
            // every product has completed: the Q ring is idle and stages the rows (4 KB per warp)
            const uint32_t stage = smem_u32(sm.q[0]) + (uint32_t)warp * 4096;
#pragma unroll 1
            for (int cc = hf * 2; cc < hf * 2 + 2; ++cc) {
                float a[32], bq[32];
                tmem_ld32(tdK + lane_off + cc * 32, a);
                tmem_ld32(tdV + lane_off + cc * 32, bq);
                tmem_wait_ld();
                store_rows_staged(p.dk, p, b, k_pos - lane, h, cc * 32, a, stage, lane);
                store_rows_staged(p.dv, p, b, k_pos - lane, h, cc * 32, bq, stage, lane);
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
//
// TMEM: S in two buffers (columns [0, 128) and [384, 512)), dP at [128, 256),
// the dQ accumulator at [256, 384).  The MMA thread keeps S two key blocks
// ahead: per block j, once dS_j is written back over dP_j it issues
//   dQ += dS_j K_j,  dP_{j+1} = dO V_{j+1}^T (over dS_j, in order),
//   S_{j+2} = Q K_{j+2}^T into the S buffer that S_j has left,
// so the math warps compute P_{j+1} from S_{j+1} (already in TMEM) while dQ_j
// and dP_{j+1} run, and only the dS phase waits for a product.  K blocks sit in
// a three-stage ring (K_j serves S_j two blocks before dQ_j), V blocks in a
// two-stage ring.
// ---------------------------------------------------------------------------
constexpr int kKStages = 3;
constexpr int kVStages = 2;
struct __align__(1024) SmemQ {
    uint8_t q[kTileBytes];
    uint8_t dout[kTileBytes];
    uint8_t k[kKStages][kTileBytes];
    uint8_t v[kVStages][kTileBytes];
    uint64_t q_full;
    uint64_t k_full[kKStages];
    uint64_t k_empty[kKStages];
    uint64_t v_full[kVStages];
    uint64_t v_empty[kVStages];
    uint64_t s_full[2];
    uint64_t dp_full;
    uint64_t ds_full;
    uint64_t acc_done;
    uint64_t mma_done;
    uint32_t tmem_base;
};
static_assert(sizeof(SmemQ) + 1024 <= 232448, "dq kernel shared memory exceeds 227 KB");
static_assert(sizeof(SmemKV) + 1024 <= 232448, "dkdv kernel shared memory exceeds 227 KB");

__global__ void __launch_bounds__(kThreads, 1)
attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
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
        for (int s = 0; s < kKStages; ++s) {
            mbar_init(&sm.k_full[s], 1);
            mbar_init(&sm.k_empty[s], 1);
        }
        for (int s = 0; s < kVStages; ++s) {
            mbar_init(&sm.v_full[s], 1);
            mbar_init(&sm.v_empty[s], 1);
        }
        mbar_init(&sm.s_full[0], 1);
        mbar_init(&sm.s_full[1], 1);
        mbar_init(&sm.dp_full, 1);
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
    const uint32_t tdP = tmem + 128, tdQ = tmem + 256;
    auto s_buf = [&](int j) { return (j & 1) ? tmem + 384 : tmem; };

    if (warp == kTmaWarp) {
        // ------------------------------ TMA producer ------------------------
        if (lane == 0) {
            mbar_arrive_expect_tx(&sm.q_full, 2 * kTileBytes);
            for (int hf = 0; hf < 2; ++hf) {
                tma_load_4d(sm.q + hf * kHalfBytes, &tmap_q, &sm.q_full, hf * 64, h, qb * kBM, b);
                tma_load_4d(sm.dout + hf * kHalfBytes, &tmap_do, &sm.q_full, hf * 64, h, qb * kBM, b);
            }
            int issued_k = 0, issued_v = 0;
            for (int j = 0; j < nk; ++j) {
                const int sk = j % kKStages, sv = j % kVStages;
                const int kt = j * kBM;
                if (!mbar_wait(&sm.k_empty[sk], ((j / kKStages) & 1) ^ 1, kSiteEmpty)) break;
                mbar_arrive_expect_tx(&sm.k_full[sk], kTileBytes);
                for (int hf = 0; hf < 2; ++hf)
                    tma_load_4d(sm.k[sk] + hf * kHalfBytes, &tmap_k, &sm.k_full[sk], hf * 64, h, kt, b);
                ++issued_k;
                if (!mbar_wait(&sm.v_empty[sv], ((j / kVStages) & 1) ^ 1, kSiteEmpty)) break;
                mbar_arrive_expect_tx(&sm.v_full[sv], kTileBytes);
                for (int hf = 0; hf < 2; ++hf)
                    tma_load_4d(sm.v[sv] + hf * kHalfBytes, &tmap_v, &sm.v_full[sv], hf * 64, h, kt, b);
                ++issued_v;
            }
            if (error_raised()) {
                mbar_wait(&sm.q_full, 0, kSiteLoad);
                for (int j = max(0, issued_k - kKStages); j < issued_k; ++j)
                    mbar_wait(&sm.k_full[j % kKStages], (j / kKStages) & 1, kSiteLoad);
                for (int j = max(0, issued_v - kVStages); j < issued_v; ++j)
                    mbar_wait(&sm.v_full[j % kVStages], (j / kVStages) & 1, kSiteLoad);
            }
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------ MMA issuer --------------------------
        if (lane == 0) {
            constexpr uint32_t idesc_ss = umma_idesc_bf16(kBM, kBM, 0, 0);
            constexpr uint32_t idesc_ts = umma_idesc_bf16(kBM, kD, 0, 1);
            const uint32_t qa = smem_u32(sm.q), da = smem_u32(sm.dout);
            // S_j = Q K_j^T into buffer j & 1 (K_j must have landed)
            auto issue_s = [&](int j) -> bool {
                const int sk = j % kKStages;
                if (!mbar_wait(&sm.k_full[sk], (j / kKStages) & 1, kSiteLoad)) return false;
                tc_fence_after();
                const uint32_t ka = smem_u32(sm.k[sk]);
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk)
                    umma_ss(s_buf(j), desc_kmajor(qa, kk), desc_kmajor(ka, kk), idesc_ss, kk > 0 ? 1u : 0u);
                umma_commit(&sm.s_full[j & 1]);
                return true;
            };
            // dP_j = dO V_j^T (V_j must have landed; its stage is free once the product completes)
            auto issue_dp = [&](int j) -> bool {
                const int sv = j % kVStages;
                if (!mbar_wait(&sm.v_full[sv], (j / kVStages) & 1, kSiteLoad)) return false;
                tc_fence_after();
                const uint32_t va = smem_u32(sm.v[sv]);
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk)
                    umma_ss(tdP, desc_kmajor(da, kk), desc_kmajor(va, kk), idesc_ss, kk > 0 ? 1u : 0u);
                umma_commit(&sm.dp_full);
                umma_commit(&sm.v_empty[sv]);
                return true;
            };
            bool ok = mbar_wait(&sm.q_full, 0, kSiteLoad);
            if (ok && nk > 0) ok = issue_s(0);
            if (ok && nk > 0) ok = issue_dp(0);
            if (ok && nk > 1) ok = issue_s(1);
            for (int j = 0; ok && j < nk; ++j) {
                if (!mbar_wait(&sm.ds_full, j & 1, kSiteP)) { ok = false; break; }
                tc_fence_after();
                // dQ += dS_j K_j  (dS: bf16 pairs over the packed columns of dP)
                const int sk = j % kKStages;
                const uint32_t ka = smem_u32(sm.k[sk]);
#pragma unroll
                for (int kk = 0; kk < kBM / 16; ++kk)
                    umma_ts(tdQ, tdP + packed_col(kk), desc_mnmajor(ka, kk), idesc_ts, (j > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&sm.k_empty[sk]);
                // dP_{j+1} after dQ_j has read dS_j from the same columns (in-order issue)
                if (j + 1 < nk && !issue_dp(j + 1)) { ok = false; break; }
                // S_{j+2} into the buffer of S_j, which the math warps have read (ds_full)
                if (j + 2 < nk && !issue_s(j + 2)) { ok = false; break; }
            }
            if (ok && nk > 0) umma_commit(&sm.acc_done);
            umma_commit(&sm.mma_done);
            mbar_wait(&sm.mma_done, 0, kSiteDone);
        }
        __syncwarp();
    } else if (warp < 8) {
        // ------------------------------ math warps --------------------------
        // thread = query row r; P then dS over the 64 keys of this warp's column
        // half in two 32-key chunks (unrolled: P stays in registers), dS written
        // over dP.
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
            // warp-uniform waits: each phase synchronises the warp
            if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[j & 1], (j >> 1) & 1, kSiteS))) { ok = false; break; }
            tc_fence_after();
            const int k0 = j * kBM;
            const bool masked = (p.causal && j == qb) || (k0 + kBM > p.T);
            const uint32_t tS = s_buf(j);
            float pr[2][32];
            // both 32-column loads in flight before the one wait
            tmem_ld32(tS + lane_off + hf * 64, pr[0]);
            tmem_ld32(tS + lane_off + hf * 64 + 32, pr[1]);
            tmem_wait_ld();
#pragma unroll
            for (int ch = 0; ch < 2; ++ch)
#pragma unroll
                for (int e = 0; e < 32; ++e) pr[ch][e] = ex2_approx(pr[ch][e] * c - lse_r);
            // Masks (the diagonal block, a partial last block) are a separate pass:
            // written inside the loop above, their per-element tests cost more
            // than the exponentials on every block.
            if (masked) {
                const int lim = (p.causal ? min(q_pos, p.T - 1) : p.T - 1) - (k0 + hf * 64);  // keys > lim are masked
#pragma unroll
                for (int ch = 0; ch < 2; ++ch)
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        if (ch * 32 + e > lim) pr[ch][e] = 0.f;
            }
            if (!__all_sync(0xffffffffu, mbar_wait(&sm.dp_full, j & 1, kSiteS))) { ok = false; break; }
            tc_fence_after();
            float dp[2][32];
            tmem_ld32(tdP + lane_off + hf * 64, dp[0]);
            tmem_ld32(tdP + lane_off + hf * 64 + 32, dp[1]);
            tmem_wait_ld();
#pragma unroll
            for (int ch = 0; ch < 2; ++ch) {
                uint32_t pd[16];
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    pd[e] = pack_bf16x2(pr[ch][2 * e] * (dp[ch][2 * e] - d_r) * p.scale,
                                        pr[ch][2 * e + 1] * (dp[ch][2 * e + 1] - d_r) * p.scale);
                tmem_st16(tdP + lane_off + hf * 64 + ch * 16, pd);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.ds_full);
        }
        bool got = ok && nk > 0 && mbar_wait(&sm.acc_done, 0, kSiteAcc);
        got = __all_sync(0xffffffffu, got);  // the staged stores synchronise the warp
        if (got) {
            tc_fence_after();
            // every product has completed: the Q tile is idle and stages the rows (4 KB per warp)
            const uint32_t stage = smem_u32(sm.q) + (uint32_t)warp * 4096;
#pragma unroll 1
            for (int cc = hf * 2; cc < hf * 2 + 2; ++cc) {
                float a[32];
                tmem_ld32(tdQ + lane_off + cc * 32, a);
                tmem_wait_ld();
                store_rows_staged(p.dq, p, b, q_pos - lane, h, cc * 32, a, stage, lane);
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

}  // namespace attn_bwd
}  // namespace dt
