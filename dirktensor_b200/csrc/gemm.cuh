// Projection GEMM for sm_100a: C[M,N] = A[M,K] . B[N,K]^T, bf16 operands,
// fp32 accumulation in TMEM, fp32 or bf16 output.
//
// Replaces the reference's projection products x . W^T
// (xt::linalg::dot(input_2d, transpose(W)), OlmoAttention.cpp:68,74,80 for
// Q/K/V and :103-105 for O).  W keeps the checkpoint's [out, in] row-major
// layout, which is exactly a K-major B operand, so no transpose is needed.
//
// Tile 128 x 256 x 64 (one 128-byte swizzle span of bf16 along K), a 4-stage
// TMA ring (48 KB per stage), one tcgen05.mma of 128x256x16 per 16-wide K
// step, accumulator in 256 TMEM columns.
//   warp 0      TMA producer
//   warp 1      MMA issuer (one thread) and TMEM owner
//   warps 2-5   epilogue: TMEM -> registers -> global (one row per thread)
// A may also be "planar": a_planes arrays [M, a_plane_k] stored back to back,
// forming A[m, p*a_plane_k + x] = plane_p[m, x].  That is the layout in which
// an all-to-all delivers a token slice of the per-head attention outputs from
// head-sharded ranks (plane = source rank), so the O projection reads it with a
// 3-D tensor map instead of a repacking pass.
#pragma once
#include "dt_common.cuh"

namespace dt {
namespace gemm {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB
constexpr int kBBytes = kBN * kBK * 2;  // 32 KB
constexpr int kThreads = 192;

struct Params {
    int M, N, K;
    void* C;            // [M, ldc] row-major
    long long ldc;      // elements
    int c_bf16;         // 0: fp32, 1: bf16
    int a_plane_k;      // 0: A is [M, K]; else A is planar with planes of this K extent
};

struct __align__(1024) Smem {
    uint8_t a[kStages][kABytes];
    uint8_t b[kStages][kBBytes];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t acc_full;
    uint64_t mma_done;
    uint32_t tmem_base;
};

enum : unsigned { kSiteEmpty = 0x21, kSiteFull, kSiteAcc, kSiteDone };

__global__ void __launch_bounds__(kThreads, 1)
gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    const Params p) {
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kBN;
    const int m0 = blockIdx.y * kBM;
    const int nk = (p.K + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        mbar_init(&sm.acc_full, 1);
        mbar_init(&sm.mma_done, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&sm.tmem_base, kBN);
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
        if (lane == 0) {
            int issued = 0;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kStages;
                const uint32_t ph = (kb / kStages) & 1;
                if (!mbar_wait(&sm.empty[s], ph ^ 1, kSiteEmpty)) break;
                mbar_arrive_expect_tx(&sm.full[s], kABytes + kBBytes);
                if (p.a_plane_k) {
                    const int plane = (kb * kBK) / p.a_plane_k;
                    tma_load_3d(sm.a[s], &tmap_a, &sm.full[s], kb * kBK - plane * p.a_plane_k, m0, plane);
                } else {
                    tma_load_2d(sm.a[s], &tmap_a, &sm.full[s], kb * kBK, m0);
                }
                tma_load_2d(sm.b[s], &tmap_b, &sm.full[s], kb * kBK, n0);
                ++issued;
            }
            if (error_raised())
                for (int kb = max(0, issued - kStages); kb < issued; ++kb)
                    mbar_wait(&sm.full[kb % kStages], (kb / kStages) & 1, kSiteFull);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(kBM, kBN, 0, 0);
            bool ok = true;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kStages;
                if (!mbar_wait(&sm.full[s], (kb / kStages) & 1, kSiteFull)) { ok = false; break; }
                tc_fence_after();
                const uint32_t a0 = smem_u32(sm.a[s]);
                const uint32_t b0 = smem_u32(sm.b[s]);
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk)
                    umma_ss(tmem, umma_desc_sw128(a0 + kk * 32, 16, 1024), umma_desc_sw128(b0 + kk * 32, 16, 1024),
                            idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&sm.empty[s]);
            }
            if (ok) umma_commit(&sm.acc_full);
            umma_commit(&sm.mma_done);
            mbar_wait(&sm.mma_done, 0, kSiteDone);
        }
        __syncwarp();
    } else {
        // epilogue warps 2..5 -> TMEM lane quarter (warp % 4)
        const int q = warp & 3;
        const int row = m0 + q * 32 + lane;
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
        if (mbar_wait(&sm.acc_full, 0, kSiteAcc)) {
            tc_fence_after();
#pragma unroll 1
            for (int cc = 0; cc < kBN / 32; ++cc) {
                float v[32];
                tmem_ld32(taddr + cc * 32, v);
                tmem_wait_ld();
                const int col = n0 + cc * 32;
                if (row < p.M && col < p.N) {
                    if (col + 32 <= p.N) {
                        if (p.c_bf16) {
                            uint4* d = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.C) +
                                                                (long long)row * p.ldc + col);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                uint4 w;
                                w.x = pack_bf16x2(v[8 * i + 0], v[8 * i + 1]);
                                w.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
                                w.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
                                w.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
                                d[i] = w;
                            }
                        } else {
                            float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.C) +
                                                                  (long long)row * p.ldc + col);
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            if (col + e < p.N) {
                                if (p.c_bf16)
                                    reinterpret_cast<__nv_bfloat16*>(p.C)[(long long)row * p.ldc + col + e] =
                                        __float2bfloat16_rn(v[e]);
                                else
                                    reinterpret_cast<float*>(p.C)[(long long)row * p.ldc + col + e] = v[e];
                            }
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kBN);
    }
}

}  // namespace gemm
}  // namespace dt
