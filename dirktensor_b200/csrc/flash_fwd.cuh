// Causal / full online-softmax attention forward for sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces the reference's flash_attention_forward (FlashAttention.cpp:24-182):
// O = softmax(scale * Q K^T + causal mask) V per (batch, head), plus the
// per-row statistics softmax_m (row max of the scaled scores) and softmax_l
// (sum of exp(s - m)) with the reference's meaning (FlashAttention.h:6-10).
//
// Operands are bf16 in the reference's token-major layout [B, T, H, D]
// (row stride H*D); TMA reads a 128-token x 64-dim box of one head per copy
// through a 4-D tensor map (D, H, T, B), so tokens past T are zero-filled and
// never cross into the next batch element.  Accumulation and softmax are fp32.
//
// CTA = one (b, h, 256-row block) work item, processed as two 128-row Q tiles
// (Q0 = rows [256c, 256c+128), Q1 = the next 128) that share every K/V tile:
//   warps 0-3  softmax warpgroup for Q0 (one thread per query row = TMEM lane)
//   warps 4-7  softmax warpgroup for Q1
//   warp 8     TMA producer (Q0, Q1 once; then K0, V0, K1, V1, ... into a ring)
//   warp 9     MMA issuer (one thread) and TMEM owner
//   warps 10-11 idle (they complete warpgroup 2; registers are granted per warpgroup)
// TMEM (512 columns x 128 lanes x 32 bit): S0 [0,128) S1 [128,256)
// O0 [256,384) O1 [384,512); P_i (bf16 pairs) overwrites the first 64 columns
// of S_i and feeds the PV product straight from TMEM.
// The MMA issue order  PV0(j), S0(j+1), PV1(j), S1(j+1)  lets the tensor core
// work on one tile while the other tile's warpgroup does its softmax; because
// tcgen05 ops of one thread complete in issue order, the commit for S_i(j+1)
// also tells softmax i that PV_i(j) has landed in O_i, so the lazy O rescale
// (done only when the running max grows by more than 2^8) needs no extra wait.
// Causal block skipping: tile i of block c visits KV tiles 0..2c+i only;
// element masks are applied on the diagonal tile and on a partial last tile.
// Grid order puts the longest (highest c) blocks first.
#pragma once
#include "dt_common.cuh"

namespace dt {
namespace attn_fwd {

constexpr int kD = 128;
constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kQTiles = 2;
constexpr int kStages = 4;
constexpr int kTileBytes = kBM * kD * 2;   // 32 KB
constexpr int kHalfBytes = kTileBytes / 2; // 128 rows x 128 B (one swizzle span of 64 bf16)
constexpr int kThreads = 384;  // 3 warpgroups: registers are granted per warpgroup
constexpr float kRescaleThreshold = 8.0f;  // log2 units
// Of every 16 column pairs of an unmasked S tile, this many compute 2^x on the
// FMA pipe (exp2_poly_pair) instead of the MUFU.  Measured on B200 with 0, 2, 4
// and 6 pairs: every step away from 0 was slower at every shape (the softmax is
// bound by its instruction stream and latency chain, not by the MUFU rate), so
// the default is 0; the path stays available for a schedule that is MUFU-bound.
#ifndef DT_FLASH_EMU_PAIRS
#define DT_FLASH_EMU_PAIRS 0
#endif
constexpr int kEmuPairs = DT_FLASH_EMU_PAIRS;

struct Params {
    int B, T, H;
    int nblk;               // work items per (b, h): blocks of qtiles * 128 rows
    int qtiles;             // Q tiles per CTA: 2 (256-row blocks), or 1 when 256-row
                            // blocks would leave SMs idle (short sequences)
    int group;              // (b, h) pairs per scheduling group (L2-resident K/V working set)
    int causal;
    float scale;            // the caller's scale (reference: 1/sqrt(head_dim))
    float scale_log2;       // scale * log2(e)
    void* out;              // [B, T, H, D] (row stride out_row_stride elements)
    int out_bf16;           // 0: fp32 output, 1: bf16 output
    long long out_row_stride;
    float* m_out;           // [B, T, H] or null
    float* l_out;           // [B, T, H] or null
    const int* seq_lens;    // [B] or null; rows t >= seq_lens[b] are written as zeros
    // Exchange mode (head-parallel path; scatter_ranks > 0): the row of global
    // token g = b*T + t is stored into rank r = g / tokens_per_rank's receive
    // buffer scatter_dst[r] (this GPU's own or a peer's, mapped over NVLink) at
    // plane scatter_plane (this rank), row g - r*tokens_per_rank; each plane is
    // [tokens_per_rank, out_row_stride].  `out` is unused then.
    int scatter_ranks;
    int scatter_plane;
    long long tokens_per_rank;
    void* scatter_dst[8];
    // fp32 Q (null: Q arrives as bf16 through tmap_q).  The softmax warps read
    // their own rows ([B, T, H, D], q_row_stride elements between tokens), round
    // them to bf16 and write the swizzled tile the tensor map would have written,
    // which removes the separate fp32 -> bf16 pass over Q.
    const float* q_f32;
    long long q_row_stride;
};

struct __align__(1024) Smem {
    uint8_t q[kQTiles][kTileBytes];
    uint8_t kv[kStages][kTileBytes];
    uint64_t q_full;
    uint64_t kv_full[kStages];
    uint64_t kv_empty[kStages];
    uint64_t s_full[kQTiles];
    uint64_t p_full[kQTiles];
    uint64_t o_full[kQTiles];
    uint64_t mma_done;
    uint32_t tmem_base;
};

// Wait-site ids reported with a timeout.
enum : unsigned { kSiteQ = 1, kSiteKvEmpty, kSiteKvFull, kSiteS, kSiteP, kSiteO, kSiteDone };

// Writes 32 consecutive output columns [col0, col0+32) of row (b, t, h), each multiplied by `mul`.
__device__ __forceinline__ void store_chunk(const Params& p, int b, int t, int h, int col0, const float* v, float mul) {
    const long long g = (long long)b * p.T + t;
    void* dst = p.out;
    long long row = g;
    if (p.scatter_ranks > 0) {
        const int r = static_cast<int>(g / p.tokens_per_rank);
        dst = p.scatter_dst[r];
        row = (long long)p.scatter_plane * p.tokens_per_rank + (g - (long long)r * p.tokens_per_rank);
    }
    const long long base = row * p.out_row_stride + (long long)h * kD + col0;
    if (p.out_bf16) {
        uint4* d4 = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dst) + base);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint4 w;
            w.x = pack_bf16x2(v[8 * i + 0] * mul, v[8 * i + 1] * mul);
            w.y = pack_bf16x2(v[8 * i + 2] * mul, v[8 * i + 3] * mul);
            w.z = pack_bf16x2(v[8 * i + 4] * mul, v[8 * i + 5] * mul);
            w.w = pack_bf16x2(v[8 * i + 6] * mul, v[8 * i + 7] * mul);
            d4[i] = w;
        }
    } else {
        float4* d4 = reinterpret_cast<float4*>(reinterpret_cast<float*>(dst) + base);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            d4[i] = make_float4(v[4 * i] * mul, v[4 * i + 1] * mul, v[4 * i + 2] * mul, v[4 * i + 3] * mul);
    }
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
attn_fwd_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                 const __grid_constant__ CUtensorMap tmap_v, const Params p) {
    pdl_enter();
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // ---- work item ------------------------------------------------------
    // (b, h) pairs are taken in groups of p.group; inside a group the blocks run
    // heaviest (highest c) first.  CTAs are dispatched in blockIdx order, so the
    // K/V of one group (group * T * 512 B) stay in L2 while its blocks run.
    const int BH = p.B * p.H;
    const int per_group = p.group * p.nblk;
    const int gi = static_cast<int>(blockIdx.x) / per_group;
    const int g0 = gi * p.group;
    const int gsz = min(p.group, BH - g0);
    const int gidx = static_cast<int>(blockIdx.x) - gi * per_group;
    const int c = p.nblk - 1 - gidx / gsz;
    const int bh = g0 + gidx % gsz;
    const int b = bh / p.H;
    const int h = bh % p.H;
    const int Tb = p.seq_lens ? min(max(p.seq_lens[b], 0), p.T) : p.T;
    const int q0 = c * (p.qtiles * kBM);
    const int nkv_all = (Tb + kBN - 1) / kBN;
    // KV tiles visited by Q tile 0 and Q tile 1 (0 when the tile starts past the sequence)
    const int n_t0 = (q0 < Tb) ? (p.causal ? min(p.qtiles * c + 1, nkv_all) : nkv_all) : 0;
    const int n_t1 = (p.qtiles > 1 && q0 + kBM < Tb) ? (p.causal ? min(2 * c + 2, nkv_all) : nkv_all) : 0;
    const int nkv = max(n_t0, n_t1);

    if (threadIdx.x == 0) {
        mbar_init(&sm.q_full, p.q_f32 ? 8 : 1);  // 8 softmax warps, or the TMA transaction
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.kv_full[s], 1);
            mbar_init(&sm.kv_empty[s], 1);
        }
        for (int i = 0; i < kQTiles; ++i) {
            mbar_init(&sm.s_full[i], 1);
            mbar_init(&sm.p_full[i], 4);
            mbar_init(&sm.o_full[i], 1);
        }
        mbar_init(&sm.mma_done, 1);
        fence_mbar_init();
    }
    if (warp == 9) {
        tmem_alloc(&sm.tmem_base, 512);
        tmem_relinquish();
    }
    if (warp == 8 && lane == 0) {
        tma_prefetch_desc(&tmap_q);
        tma_prefetch_desc(&tmap_k);
        tma_prefetch_desc(&tmap_v);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    if (warp == 8) {
        // ------------------------------ TMA producer ------------------------
        if (lane == 0 && nkv > 0) {
            if (!p.q_f32) {
                mbar_arrive_expect_tx(&sm.q_full, p.qtiles * kTileBytes);
                for (int i = 0; i < p.qtiles; ++i)
                    for (int hf = 0; hf < 2; ++hf)
                        tma_load_4d(sm.q[i] + hf * kHalfBytes, &tmap_q, &sm.q_full, hf * 64, h, q0 + i * kBM, b);
            }
            int issued = 0;
            for (int L = 0; L < 2 * nkv; ++L) {
                const int s = L % kStages;
                const uint32_t ph = (L / kStages) & 1;
                if (!mbar_wait_sleep(&sm.kv_empty[s], ph ^ 1, kSiteKvEmpty)) break;
                mbar_arrive_expect_tx(&sm.kv_full[s], kTileBytes);
                const int kt = (L >> 1) * kBN;
                for (int hf = 0; hf < 2; ++hf) {
                    if (L & 1) tma_load_4d(sm.kv[s] + hf * kHalfBytes, &tmap_v, &sm.kv_full[s], hf * 64, h, kt, b);
                    else tma_load_4d(sm.kv[s] + hf * kHalfBytes, &tmap_k, &sm.kv_full[s], hf * 64, h, kt, b);
                }
                ++issued;
            }
            if (error_raised()) {
                // Drain copies still in flight before the CTA exits.
                for (int L = max(0, issued - kStages); L < issued; ++L)
                    mbar_wait_sleep(&sm.kv_full[L % kStages], (L / kStages) & 1, kSiteKvFull);
                mbar_wait_sleep(&sm.q_full, 0, kSiteQ);
            }
        }
    } else if (warp == 9) {
        // ------------------------------ MMA issuer --------------------------
        if (lane == 0 && nkv > 0) {
            constexpr uint32_t idesc_qk = umma_idesc_bf16(kBM, kBN, 0, 0);
            constexpr uint32_t idesc_pv = umma_idesc_bf16(kBM, kD, 0, 1);
            bool ok = mbar_wait_sleep(&sm.q_full, 0, kSiteQ);
            auto stage_of = [](int L) { return L % kStages; };
            auto phase_of = [](int L) { return (uint32_t)((L / kStages) & 1); };
            auto issue_s = [&](int i, int L) {
                const uint32_t kaddr = smem_u32(sm.kv[stage_of(L)]);
                const uint32_t qaddr = smem_u32(sm.q[0]) + (uint32_t)i * kTileBytes;
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
                    umma_ss(tmem + i * 128, umma_desc_sw128(qaddr + off, 16, 1024),
                            umma_desc_sw128(kaddr + off, 16, 1024), idesc_qk, kk > 0 ? 1u : 0u);
                }
                umma_commit(&sm.s_full[i]);
            };
            auto issue_pv = [&](int i, int L, bool acc) {
                const uint32_t vaddr = smem_u32(sm.kv[stage_of(L)]);
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk) {
                    // V is MN-major for this product: 64-dim halves kHalfBytes apart (LBO),
                    // 8-key groups 1024 B apart (SBO); 16 keys per instruction.
                    umma_ts(tmem + 256 + i * 128, tmem + i * 128 + kk * 8,
                            umma_desc_sw128(vaddr + kk * 2048, kHalfBytes, 1024), idesc_pv,
                            (acc || kk > 0) ? 1u : 0u);
                }
            };
            if (ok) ok = mbar_wait_sleep(&sm.kv_full[stage_of(0)], phase_of(0), kSiteKvFull);
            if (ok) {
                tc_fence_after();
                if (n_t0 > 0) issue_s(0, 0);
                if (n_t1 > 0) issue_s(1, 0);
                umma_commit(&sm.kv_empty[stage_of(0)]);
            }
            for (int j = 0; ok && j < nkv; ++j) {
                const int LV = 2 * j + 1, LK = 2 * j + 2;
                const bool next_k = (j + 1) < nkv;
                ok = mbar_wait_sleep(&sm.kv_full[stage_of(LV)], phase_of(LV), kSiteKvFull);
                if (ok && next_k) ok = mbar_wait_sleep(&sm.kv_full[stage_of(LK)], phase_of(LK), kSiteKvFull);
                if (!ok) break;
                tc_fence_after();
                for (int i = 0; i < kQTiles; ++i) {
                    const int ni = (i == 0) ? n_t0 : n_t1;
                    if (j >= ni) continue;
                    if (!mbar_wait_sleep(&sm.p_full[i], j & 1, kSiteP)) { ok = false; break; }
                    tc_fence_after();
                    issue_pv(i, LV, j > 0);
                    if (j + 1 < ni) issue_s(i, LK);
                    else umma_commit(&sm.o_full[i]);
                }
                if (!ok) break;
                umma_commit(&sm.kv_empty[stage_of(LV)]);
                if (next_k) umma_commit(&sm.kv_empty[stage_of(LK)]);
            }
            // All issued tcgen05 work must be complete before TMEM is released.
            umma_commit(&sm.mma_done);
            mbar_wait_sleep(&sm.mma_done, 0, kSiteDone);
        }
        __syncwarp();
    } else if (warp < 8) {
        // --------------------------- softmax warpgroups ---------------------
        if (p.q_f32) {
            // This warp's 32 rows of Q tile (warp >> 2), fp32 -> bf16, in the
            // 128-byte-swizzled K-major layout of a TMA load: row r of a 64-dim
            // half at r * 128, its 16-byte chunk c at position c ^ (r & 7).  One
            // coalesced 512-byte row per load instruction (lane = 4 dims), all 32
            // rows' loads in flight at once (with 8 in flight the four
            // round trips to DRAM per CTA cost more than the cast they replace);
            // rows at or past T are zeros, as the tensor map fills them.
            const uint32_t qs = smem_u32(sm.q[warp >> 2]);
            const int chunk = lane >> 1;  // 16-byte chunk (8 dims) of this lane's 4 dims
            const uint32_t col = (uint32_t)(chunk >> 3) * kHalfBytes + (uint32_t)(lane & 1) * 8;
            // (a disabled second tile loads nothing)
#pragma unroll 32
            for (int rr = 0; rr < 32 && (warp >> 2) < p.qtiles; ++rr) {
                const int row = (warp & 3) * 32 + rr;
                const int t = q0 + (warp >> 2) * kBM + row;
                float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
                if (t < p.T)
                    x = __ldg(reinterpret_cast<const float4*>(p.q_f32 + ((long long)b * p.T + t) * p.q_row_stride +
                                                              (long long)h * kD) + lane);
                const uint32_t addr = qs + col + (uint32_t)row * 128 + ((uint32_t)((chunk & 7) ^ (row & 7)) << 4);
                asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(addr), "r"(pack_bf16x2(x.x, x.y)),
                             "r"(pack_bf16x2(x.z, x.w))
                             : "memory");
            }
            // generic-proxy stores become visible to the tensor cores' reads
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.q_full);
        }
        const int i = warp >> 2;          // Q tile
        const int r = (warp & 3) * 32 + lane;
        const int qt = q0 + i * kBM;
        const int q_pos = qt + r;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tS = tmem + lane_off + i * 128;
        const uint32_t tO = tmem + lane_off + 256 + i * 128;
        const int n = (i == 0) ? n_t0 : n_t1;
        float m_run = -INFINITY, l_run = 0.f, mx = -INFINITY;
        bool ok = true;
        for (int j = 0; j < n; ++j) {
            // warp-uniform, since the step synchronises the warp (__any_sync, __syncwarp)
            if (!__all_sync(0xffffffffu, mbar_wait_sleep(&sm.s_full[i], j & 1, kSiteS))) { ok = false; break; }
            tc_fence_after();
            float s[128];
            tmem_ld32(tS + 0, *reinterpret_cast<float(*)[32]>(s + 0));
            tmem_ld32(tS + 32, *reinterpret_cast<float(*)[32]>(s + 32));
            tmem_ld32(tS + 64, *reinterpret_cast<float(*)[32]>(s + 64));
            tmem_ld32(tS + 96, *reinterpret_cast<float(*)[32]>(s + 96));
            tmem_wait_ld();
            const int k0 = j * kBN;
            const bool diag = p.causal && (k0 + kBN - 1 > qt);
            const bool tail = (k0 + kBN > Tb);
            if (diag || tail) {
                const int lim = p.causal ? min(q_pos, Tb - 1) : (Tb - 1);
#pragma unroll
                for (int e = 0; e < 128; ++e)
                    if (k0 + e > lim) s[e] = -INFINITY;
            }
            // Row max as 8 independent chains over 16-column slices, then a short
            // combine: a single 64-deep chain of dependent max ops is latency-bound.
            float pm[8];
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                float a = fmax3(s[16 * g], s[16 * g + 1], s[16 * g + 2]);
#pragma unroll
                for (int e = 3; e < 15; e += 2) a = fmax3(a, s[16 * g + e], s[16 * g + e + 1]);
                pm[g] = fmaxf(a, s[16 * g + 15]);
            }
            const float rmax = fmaxf(fmax3(pm[0], pm[1], pm[2]), fmax3(fmax3(pm[3], pm[4], pm[5]), pm[6], pm[7]));
            mx = fmaxf(mx, rmax);
            const float m_cand = rmax * p.scale_log2;
            float alpha = 1.f;
            if (j == 0) {
                m_run = m_cand;
            } else {
                const bool need = m_cand > m_run + kRescaleThreshold;
                if (__any_sync(0xffffffffu, need)) {
                    if (need) {
                        alpha = ex2_approx(m_run - m_cand);
                        m_run = m_cand;
                    }
#pragma unroll 1
                    for (int cc = 0; cc < 8; ++cc) {
                        float o[16];
                        tmem_ld16(tO + cc * 16, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 16; ++e) o[e] *= alpha;
                        tmem_st16(tO + cc * 16, *reinterpret_cast<uint32_t(*)[16]>(o));
                    }
                }
            }
            // p = 2^(s*scale*log2e - m): the scale-subtract and the row sum run as
            // packed f32x2 pairs; ex2 stays per element (MUFU).
            const uint64_t c2 = f2_pack(p.scale_log2, p.scale_log2);
            const uint64_t nm2 = f2_pack(-m_run, -m_run);
            // one packed partial sum per 32-column chunk: four independent chains
            uint64_t sum2[4] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f), f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
            const bool masked = diag || tail;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                uint32_t pk[16];
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    float x0, x1, p0, p1;
                    f2_unpack(f2_fma(f2_pack(s[cc * 32 + 2 * e], s[cc * 32 + 2 * e + 1]), c2, nm2), x0, x1);
                    if (e >= 16 - kEmuPairs && !masked) {
                        exp2_poly_pair(x0, x1, p0, p1);
                    } else {
                        p0 = ex2_approx(x0);
                        p1 = ex2_approx(x1);
                    }
                    sum2[cc] = f2_add(sum2[cc], f2_pack(p0, p1));
                    pk[e] = pack_bf16x2(p0, p1);
                }
                tmem_st16(tS + cc * 16, pk);
            }
            float sum_lo, sum_hi;
            f2_unpack(f2_add(f2_add(sum2[0], sum2[1]), f2_add(sum2[2], sum2[3])), sum_lo, sum_hi);
            const float sum = sum_lo + sum_hi;
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.p_full[i]);
            l_run = l_run * alpha + sum;
        }
        // ---- epilogue: O / l and the statistics -------------------------
        // Rows past the sequence length (varlen padding) are written as zeros; a
        // disabled second tile (qtiles == 1) owns no rows.
        const bool row_in = i < p.qtiles && q_pos < p.T;
        const bool row_valid = q_pos < Tb;
        bool have_o = false;
        if (n > 0 && ok) have_o = mbar_wait_sleep(&sm.o_full[i], 0, kSiteO);
        // the staged epilogues below synchronise the warp: take them only if every lane
        // saw the accumulator (a wait that timed out on some lane is already reported)
        have_o = __all_sync(0xffffffffu, have_o);
        if (have_o && p.out_bf16) {
            // bf16 rows leave through shared memory so that global (or peer)
            // stores are coalesced: each warp stages its 32 rows (256 B each) in
            // its quarter of this tile's Q buffer -- idle now, since o_full
            // follows every S_i product that read it -- then writes two whole
            // rows (512 contiguous bytes) per instruction.  Warp-local only.
            tc_fence_after();
            const float inv_l = (l_run > 0.f) ? 1.f / l_run : 0.f;
            const float mul = row_valid ? inv_l : 0.f;
            const uint32_t stage = smem_u32(sm.q[i]) + (uint32_t)(warp & 3) * 8192;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                float o[32];
                tmem_ld32(tO + cc * 32, o);
                tmem_wait_ld();
#pragma unroll
                for (int m = 0; m < 4; ++m) {  // 16-byte chunk 4cc+m of this row, XOR-swizzled by row
                    const uint32_t chunk = (uint32_t)(4 * cc + m) ^ (uint32_t)(lane & 15);
                    st_shared_v4(stage + (uint32_t)lane * 256 + chunk * 16,
                                 pack_bf16x2(o[8 * m + 0] * mul, o[8 * m + 1] * mul),
                                 pack_bf16x2(o[8 * m + 2] * mul, o[8 * m + 3] * mul),
                                 pack_bf16x2(o[8 * m + 4] * mul, o[8 * m + 5] * mul),
                                 pack_bf16x2(o[8 * m + 6] * mul, o[8 * m + 7] * mul));
                }
            }
            __syncwarp();
#pragma unroll 4
            for (int step = 0; step < 16; ++step) {
                const int rr = 2 * step + (lane >> 4);            // row within this warp's 32
                const uint32_t chunk = (uint32_t)(lane & 15);
                const int t = qt + (warp & 3) * 32 + rr;
                uint32_t a, bb, c2, d;
                asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                             : "=r"(a), "=r"(bb), "=r"(c2), "=r"(d)
                             : "r"(stage + (uint32_t)rr * 256 + ((chunk ^ (uint32_t)(rr & 15)) << 4)));
                if (t < p.T) {
                    const long long g = (long long)b * p.T + t;
                    void* dst = p.out;
                    long long row = g;
                    if (p.scatter_ranks > 0) {
                        const int rk = static_cast<int>(g / p.tokens_per_rank);
                        dst = p.scatter_dst[rk];
                        row = (long long)p.scatter_plane * p.tokens_per_rank + (g - (long long)rk * p.tokens_per_rank);
                    }
                    uint4* d4 = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dst) + row * p.out_row_stride +
                                                         (long long)h * kD) + chunk;
                    *d4 = make_uint4(a, bb, c2, d);
                }
            }
        } else if (have_o && p.scatter_ranks == 0) {
            // fp32 rows leave through the same quarter of the Q buffer, 64 columns (256 B
            // of each row) at a time: each store instruction then writes two whole
            // 256-byte row segments instead of 32 scattered 16-byte pieces.
            tc_fence_after();
            const float inv_l = (l_run > 0.f) ? 1.f / l_run : 0.f;
            const float mul = row_valid ? inv_l : 0.f;
            const uint32_t stage = smem_u32(sm.q[i]) + (uint32_t)(warp & 3) * 8192;
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
#pragma unroll
                for (int c2 = 0; c2 < 2; ++c2) {
                    float o[32];
                    tmem_ld32(tO + half * 64 + c2 * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int m = 0; m < 8; ++m) {  // 16-byte chunk 8*c2+m of this row, XOR-swizzled by row
                        const uint32_t chunk = (uint32_t)(8 * c2 + m) ^ (uint32_t)(lane & 15);
                        st_shared_v4(stage + (uint32_t)lane * 256 + chunk * 16, __float_as_uint(o[4 * m] * mul),
                                     __float_as_uint(o[4 * m + 1] * mul), __float_as_uint(o[4 * m + 2] * mul),
                                     __float_as_uint(o[4 * m + 3] * mul));
                    }
                }
                __syncwarp();
#pragma unroll 4
                for (int step = 0; step < 16; ++step) {
                    const int rr = 2 * step + (lane >> 4);  // row within this warp's 32
                    const uint32_t chunk = (uint32_t)(lane & 15);
                    const int t = qt + (warp & 3) * 32 + rr;
                    float4 x;
                    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                                 : "=f"(x.x), "=f"(x.y), "=f"(x.z), "=f"(x.w)
                                 : "r"(stage + (uint32_t)rr * 256 + ((chunk ^ (uint32_t)(rr & 15)) << 4)));
                    if (t < p.T)
                        *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) +
                                                   ((long long)b * p.T + t) * p.out_row_stride + (long long)h * kD +
                                                   half * 64 + chunk * 4) = x;
                }
                __syncwarp();  // the next half reuses the stage
            }
        } else if (have_o) {
            tc_fence_after();
            const float inv_l = (l_run > 0.f) ? 1.f / l_run : 0.f;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                float o[32];
                tmem_ld32(tO + cc * 32, o);
                tmem_wait_ld();
                if (row_in) store_chunk(p, b, q_pos, h, cc * 32, o, row_valid ? inv_l : 0.f);
            }
        } else if (n == 0 && row_in) {
            float z[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) z[e] = 0.f;
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) store_chunk(p, b, q_pos, h, cc * 32, z, 0.f);
        }
        if (row_in && (have_o || n == 0)) {
            const long long sidx = ((long long)b * p.T + q_pos) * p.H + h;
            float m_o = 0.f, l_o = 0.f;
            if (have_o && row_valid) {
                // m: max of the scaled scores (natural units); l = sum exp(s - m),
                // converted from the kernel's lazily-updated base-2 running max.
                m_o = mx * p.scale;
                l_o = l_run * ex2_approx(m_run - mx * p.scale_log2);
            }
            if (p.m_out) p.m_out[sidx] = m_o;
            if (p.l_out) p.l_out[sidx] = l_o;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace attn_fwd
}  // namespace dt
