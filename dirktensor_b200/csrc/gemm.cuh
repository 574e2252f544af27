// Projection GEMM for sm_100a: C[M,N] = A[M,K] . B[N,K]^T, bf16 operands,
// fp32 accumulation in TMEM, fp32 or bf16 output.
//
// Replaces the reference's projection products x . W^T
// (xt::linalg::dot(input_2d, transpose(W)), OlmoAttention.cpp:68,74,80 for
// Q/K/V and :103-105 for O).  W keeps the checkpoint's [out, in] row-major
// layout, which is exactly a K-major B operand, so no transpose is needed.
//
// Persistent kernel: one CTA per SM walks the 128 x 256 output tiles
// (tile t, t + gridDim.x, ...; in the order tile_m / tile_n give, below).
// 128x256x16 tcgen05.mma per 16-wide K step.  Two accumulators of 256 TMEM
// columns alternate between tiles, so the epilogue of tile i (TMEM ->
// registers -> global) runs while the MMAs of tile i+1 proceed.
//   warp 0      TMA producer
//   warp 1      MMA issuer (one thread) and TMEM owner
//   warps 2-5   epilogue (one output row per thread, TMEM lane quarter = warp % 4)
// Epilogue kSwiGLU (the MLP's gate/up product, OlmoMlp.cpp:38-52): B holds the
// gate and up weights interleaved in 128-row blocks, so accumulator columns
// [0,128) of a tile are gate and [128,256) the matching up columns; the
// epilogue writes silu(gate) * up = gate / (1 + exp(-gate)) * up as bf16 into
// output columns [128 n, 128 n + 128) (C has N/2 columns).
// A may also be "planar": a_planes arrays [M, a_plane_k] stored back to back,
// forming A[m, p*a_plane_k + x] = plane_p[m, x].  That is the layout in which
// an all-to-all delivers a token slice of the per-head attention outputs from
// head-sharded ranks (plane = source rank), so the O projection reads it with a
// 3-D tensor map instead of a repacking pass.
// Either operand may instead be MN-major (a_mn / b_mn): stored [K, M] (or
// [K, N]) row-major, i.e. the transposed product the training path needs --
// dW = dY^T X and dX = dY W (OlmoAttention.cpp:201-205, 207, 250-267, 278-298)
// read the row-major activations and weights directly.  An MN-major tile is two
// (A) or BN/64 (B) 64-wide column strips of 64 K-rows each, loaded by 64 x 64
// TMA boxes; the UMMA descriptor steps 16 K-rows (2 KB) per instruction with the
// strips 8 KB apart.  Epilogue kAccum adds the product to an fp32 C (the
// reference's beta = 1 gradient accumulation).
#pragma once
#include "dt_common.cuh"

namespace dt {
namespace gemm {

constexpr int kBM = 128;
constexpr int kBN = 256;                // default tile width; kNarrowBN for few-tile problems
constexpr int kNarrowBN = 128;
constexpr int kBK = 64;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB
constexpr int kThreads = 192;
constexpr int kAccs = 2;                // TMEM accumulators (2 x BN columns)
// stages that fit with a 128 x BN tile: 4 x 48 KB (BN 256) or 6 x 32 KB (BN 128)
template <int BN>
struct Cfg {
    static constexpr int kStages = BN == 256 ? 4 : 6;
    static constexpr int kBBytes = BN * kBK * 2;
};

struct Params {
    int M, N, K;
    void* C;            // [M, ldc] row-major
    long long ldc;      // elements
    int c_bf16;         // 0: fp32, 1: bf16
    int a_plane_k;      // 0: A is [M, K]; else A is planar with planes of this K extent
    int tiles_n;        // ceil(N / kBN)
    int num_tiles;      // tiles_m * tiles_n
    int epilogue;       // kStore or kSwiGLU
    // Right-padded batches (optional): rows are (sequence, position) with
    // seq_T positions per sequence; a tile whose rows all lie at positions
    // >= seq_lens[sequence] is padding and is skipped (zeros are written when
    // pad_zero is set).  Only used when tiles never straddle two sequences.
    const int* seq_lens;
    int seq_T;
    int pad_zero;
    int a_mn;           // 1: A stored [K, M] row-major (M contiguous)
    int b_mn;           // 1: B stored [K, N] row-major (N contiguous)
    int tiles_m;        // ceil(M / tile rows)
    int m_fastest;      // tile order: 0 = N varies fastest, 1 = M varies fastest
    // Split output (optional, C2 != null): columns >= c2_col0 (a multiple of 32) go
    // to C2 as bf16, [M, ldc2] row-major from column c2_col0 on; the rest to C.
    // The QKV projection writes q and k in fp32 for the norm and v straight in bf16.
    void* C2;
    long long ldc2;
    int c2_col0;
};

// Tile t's (row-tile, column-tile) in the persistent walk.  The order keeps the
// larger operand's panel fixed while consecutive CTAs sweep the smaller one
// (which then stays in L2): with N fastest, the CTAs of a wave share one A row
// panel and B is re-read per row band; with M fastest (chosen when N > M, e.g.
// the LM head's 100352 x 2048 weight), they share one B panel and read it once.
__device__ __forceinline__ int tile_m(const Params& p, int t) { return p.m_fastest ? t % p.tiles_m : t / p.tiles_n; }
__device__ __forceinline__ int tile_n(const Params& p, int t) { return p.m_fastest ? t / p.tiles_m : t % p.tiles_n; }

// True when rows [m0, m0 + rows) all lie in one sequence's right padding.
__device__ __forceinline__ bool tile_is_padding(const Params& p, int m0) {
    if (!p.seq_lens) return false;
    const int b = m0 / p.seq_T;
    return (m0 - b * p.seq_T) >= p.seq_lens[b];
}

enum Epilogue : int { kStore = 0, kSwiGLU = 1, kAccum = 2 };

template <int BN>
struct __align__(1024) SmemT {
    static constexpr int kStages = Cfg<BN>::kStages;
    uint8_t a[kStages][kABytes];
    uint8_t b[kStages][Cfg<BN>::kBBytes];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t acc_full[kAccs];
    uint64_t acc_empty[kAccs];
    uint64_t mma_done;
    uint32_t tmem_base;
    alignas(128) float stage[4][32 * 32];  // epilogue: one 32 x 32 fp32 block per epilogue warp
};
using Smem = SmemT<kBN>;

enum : unsigned { kSiteEmpty = 0x21, kSiteFull, kSiteAcc, kSiteDone, kSiteAccEmpty };

__device__ __forceinline__ void store_chunk(const Params& p, int row, int col, const float (&v)[32]) {
    if (row >= p.M || col >= p.N) return;
    if (p.C2 != nullptr && col >= p.c2_col0) {
        __nv_bfloat16* base = reinterpret_cast<__nv_bfloat16*>(p.C2) + (long long)row * p.ldc2 + (col - p.c2_col0);
        if (col + 32 <= p.N) {
            uint4* d = reinterpret_cast<uint4*>(base);
#pragma unroll
            for (int i = 0; i < 4; ++i)
                d[i] = make_uint4(pack_bf16x2(v[8 * i + 0], v[8 * i + 1]), pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                                  pack_bf16x2(v[8 * i + 4], v[8 * i + 5]), pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
        } else {
#pragma unroll
            for (int e = 0; e < 32; ++e)
                if (col + e < p.N) base[e] = __float2bfloat16_rn(v[e]);
        }
        return;
    }
    if (col + 32 <= p.N) {
        if (p.c_bf16) {
            uint4* d = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.C) + (long long)row * p.ldc + col);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint4 w;
                w.x = pack_bf16x2(v[8 * i + 0], v[8 * i + 1]);
                w.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
                w.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
                w.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
                d[i] = w;
            }
        } else if (p.epilogue == kAccum) {
            float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.C) + (long long)row * p.ldc + col);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 o = d[i];
                d[i] = make_float4(o.x + v[4 * i], o.y + v[4 * i + 1], o.z + v[4 * i + 2], o.w + v[4 * i + 3]);
            }
        } else {
            float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.C) + (long long)row * p.ldc + col);
#pragma unroll
            for (int i = 0; i < 8; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
    } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            if (col + e < p.N) {
                if (p.c_bf16)
                    reinterpret_cast<__nv_bfloat16*>(p.C)[(long long)row * p.ldc + col + e] = __float2bfloat16_rn(v[e]);
                else if (p.epilogue == kAccum)
                    reinterpret_cast<float*>(p.C)[(long long)row * p.ldc + col + e] += v[e];
                else
                    reinterpret_cast<float*>(p.C)[(long long)row * p.ldc + col + e] = v[e];
            }
        }
    }
}

// True when the fp32 columns [col, col + 32) leave through store_rows_f32_staged
// (warp-uniform: depends on the column and the parameters only).
__device__ __forceinline__ bool staged_f32(const Params& p, int col) {
    return p.epilogue == kStore && !p.c_bf16 && (p.C2 == nullptr || col < p.c2_col0) && col + 32 <= p.N;
}

// Coalesced store of a warp's 32 rows x 32 fp32 columns (lane i holds row row0 + i).
// The block passes through this warp's 4 KB of shared memory -- 16-byte chunk j of
// row r at position j ^ (r & 7), so that both the row-wise writes and the
// column-wise reads spread over all banks -- and each store instruction then
// writes four whole 128-byte row segments instead of 32 scattered 16-byte pieces.
// Rows >= M are skipped.
__device__ __forceinline__ void store_rows_f32_staged(const Params& p, uint32_t stage, int row0, int col,
                                                      const float (&v)[32], int lane) {
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
        if (row0 + r < p.M)
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.C) + (long long)(row0 + r) * p.ldc + col + 4 * j) = x;
    }
    __syncwarp();  // the next block reuses the stage
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    const Params p) {
    pdl_enter();
    constexpr int kStages = Cfg<BN>::kStages;
    constexpr int kBBytes = Cfg<BN>::kBBytes;
    extern __shared__ uint8_t smem_raw[];
    SmemT<BN>& sm = *reinterpret_cast<SmemT<BN>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nk = (p.K + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        for (int a = 0; a < kAccs; ++a) {
            mbar_init(&sm.acc_full[a], 1);
            mbar_init(&sm.acc_empty[a], 4);  // one arrive per epilogue warp
        }
        mbar_init(&sm.mma_done, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&sm.tmem_base, kAccs * BN);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------
        if (lane == 0) {
            int kit = 0;  // k-blocks issued by this CTA (ring position)
            bool ok = true;
            for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
                const int m0 = tile_m(p, t) * kBM;
                const int n0 = tile_n(p, t) * BN;
                if (tile_is_padding(p, m0)) continue;
                for (int kb = 0; kb < nk; ++kb, ++kit) {
                    const int s = kit % kStages;
                    if (!mbar_wait(&sm.empty[s], ((kit / kStages) & 1) ^ 1, kSiteEmpty)) { ok = false; break; }
                    mbar_arrive_expect_tx(&sm.full[s], kABytes + kBBytes);
                    if (p.a_mn) {
                        for (int a = 0; a < kBM / 64; ++a)
                            tma_load_2d(sm.a[s] + a * 8192, &tmap_a, &sm.full[s], m0 + 64 * a, kb * kBK);
                    } else if (p.a_plane_k) {
                        const int plane = (kb * kBK) / p.a_plane_k;
                        tma_load_3d(sm.a[s], &tmap_a, &sm.full[s], kb * kBK - plane * p.a_plane_k, m0, plane);
                    } else {
                        tma_load_2d(sm.a[s], &tmap_a, &sm.full[s], kb * kBK, m0);
                    }
                    if (p.b_mn) {
                        for (int a = 0; a < BN / 64; ++a)
                            tma_load_2d(sm.b[s] + a * 8192, &tmap_b, &sm.full[s], n0 + 64 * a, kb * kBK);
                    } else {
                        tma_load_2d(sm.b[s], &tmap_b, &sm.full[s], kb * kBK, n0);
                    }
                }
            }
            if (!ok)  // drain copies still in flight before the CTA exits
                for (int k = max(0, kit - kStages); k < kit; ++k)
                    mbar_wait(&sm.full[k % kStages], (k / kStages) & 1, kSiteFull);
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer --------------------------
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_bf16(kBM, BN, p.a_mn, p.b_mn);
            int kit = 0, it = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
                if (tile_is_padding(p, tile_m(p, t) * kBM)) continue;
                const int acc = it & 1;
                const uint32_t empty_phase = ((it >> 1) & 1) ^ 1;
                ++it;
                // the epilogue must have drained this accumulator (used two tiles ago)
                if (!mbar_wait(&sm.acc_empty[acc], empty_phase, kSiteAccEmpty)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d = tmem + acc * BN;
                for (int kb = 0; kb < nk; ++kb, ++kit) {
                    const int s = kit % kStages;
                    if (!mbar_wait(&sm.full[s], (kit / kStages) & 1, kSiteFull)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sm.a[s]);
                    const uint32_t b0 = smem_u32(sm.b[s]);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        const uint64_t da = p.a_mn ? umma_desc_sw128(a0 + kk * 2048, 8192, 1024)
                                                   : umma_desc_sw128(a0 + kk * 32, 16, 1024);
                        const uint64_t db = p.b_mn ? umma_desc_sw128(b0 + kk * 2048, 8192, 1024)
                                                   : umma_desc_sw128(b0 + kk * 32, 16, 1024);
                        umma_ss(d, da, db, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(&sm.empty[s]);
                }
                if (ok) umma_commit(&sm.acc_full[acc]);
            }
            umma_commit(&sm.mma_done);
            mbar_wait(&sm.mma_done, 0, kSiteDone);
        }
        __syncwarp();
    } else {
        // -------------------------------- epilogue --------------------------
        const int q = warp & 3;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        int it = 0;
        for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
            const int row = tile_m(p, t) * kBM + q * 32 + lane;
            const int n0 = tile_n(p, t) * BN;
            if (tile_is_padding(p, tile_m(p, t) * kBM)) {
                if (p.pad_zero && p.epilogue == kStore) {
                    float z[32];
#pragma unroll
                    for (int e = 0; e < 32; ++e) z[e] = 0.f;
#pragma unroll 1
                    for (int cc = 0; cc < BN / 32; ++cc) store_chunk(p, row, n0 + cc * 32, z);
                }
                continue;
            }
            const int acc = it & 1;
            const uint32_t acc_phase = (it >> 1) & 1;
            ++it;
            // warp-uniform: the staged stores below synchronise the warp (a lane whose
            // wait expired has recorded the error; the whole warp stops)
            if (!__all_sync(0xffffffffu, mbar_wait(&sm.acc_full[acc], acc_phase, kSiteAcc))) break;
            tc_fence_after();
            const uint32_t taddr = tmem + lane_off + acc * BN;
            if (p.epilogue == kSwiGLU) {
                const int oc0 = tile_n(p, t) * (BN / 2);
#pragma unroll 1
                for (int cc = 0; cc < BN / 64; ++cc) {
                    float g[32], u[32];
                    tmem_ld32(taddr + cc * 32, g);
                    tmem_ld32(taddr + BN / 2 + cc * 32, u);
                    tmem_wait_ld();
                    const int oc = oc0 + cc * 32;
                    if (row < p.M && oc + 32 <= p.N / 2) {
                        uint4* d = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.C) +
                                                            (long long)row * p.ldc + oc);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            float a[8];
#pragma unroll
                            for (int e = 0; e < 8; ++e) {
                                const float x = g[8 * i + e];
                                a[e] = x / (1.f + __expf(-x)) * u[8 * i + e];
                            }
                            uint4 w;
                            w.x = pack_bf16x2(a[0], a[1]);
                            w.y = pack_bf16x2(a[2], a[3]);
                            w.z = pack_bf16x2(a[4], a[5]);
                            w.w = pack_bf16x2(a[6], a[7]);
                            d[i] = w;
                        }
                    }
                }
            } else {
                const uint32_t stage = smem_u32(sm.stage[q]);
#pragma unroll 1
                for (int cc = 0; cc < BN / 32; ++cc) {
                    float v[32];
                    tmem_ld32(taddr + cc * 32, v);
                    tmem_wait_ld();
                    if (staged_f32(p, n0 + cc * 32))
                        store_rows_f32_staged(p, stage, row - lane, n0 + cc * 32, v, lane);
                    else
                        store_chunk(p, row, n0 + cc * 32, v);
                }
            }
            // accumulator drained: hand it back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.acc_empty[acc]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kAccs * BN);
    }
}

}  // namespace gemm
}  // namespace dt
