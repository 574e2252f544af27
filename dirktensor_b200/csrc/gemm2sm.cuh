// Projection GEMM on SM pairs (tcgen05 cta_group::2): C[M,N] = A[M,K] . B[N,K]^T,
// bf16 operands, fp32 accumulation in TMEM.  Same contract as gemm.cuh (store
// and SwiGLU epilogues, planar A), for large M.
//
// A cluster of two CTAs on two SMs computes a 256 x 256 output tile per step:
// CTA r loads A rows [m0 + 128 r, +128) and B rows [n0 + 128 r, +128) into its
// own shared memory (TMA, no cluster-wide copies); the leader CTA (rank 0)
// issues one 256x256x16 tcgen05.mma per K step, which reads both CTAs' tiles
// and leaves rows [128 r, 128 r + 128) of the product in CTA r's TMEM.  Per SM
// that is 32 KB of operands per 64-wide K step instead of 48 KB for a 128 x 256
// tile on one SM, so the L2 -> shared memory traffic per FLOP drops by a third.
// Both CTAs' loads complete on the leader's barrier; the leader's commits reach
// both CTAs' barriers (tcgen05.commit with a CTA mask); each CTA drains its own
// TMEM rows and reports back to the leader's accumulator barrier.
//   warp 0      TMA producer (both CTAs)
//   warp 1      MMA issuer (leader CTA) and TMEM owner (both CTAs, cta_group::2)
//   warps 2-5   epilogue (both CTAs)
#pragma once
#include "dt_common.cuh"
#include "gemm.cuh"

namespace dt {
namespace gemm2 {

constexpr int kBM = 256;   // rows per cluster tile (128 per CTA)
constexpr int kBN = 256;   // columns per cluster tile (B rows: 128 loaded per CTA)
constexpr int kBK = 64;
constexpr int kStages = 6;
constexpr int kHalf = 128;
constexpr int kABytes = kHalf * kBK * 2;  // 16 KB
constexpr int kBBytes = kHalf * kBK * 2;  // 16 KB
constexpr int kThreads = 192;
constexpr int kAccs = 2;

using Params = dt::gemm::Params;  // tiles_n counts kBN-wide tiles, num_tiles cluster tiles

struct __align__(1024) Smem {
    uint8_t a[kStages][kABytes];
    uint8_t b[kStages][kBBytes];
    uint64_t full[kStages];       // leader: both CTAs' stage s landed
    uint64_t empty[kStages];      // both: stage s consumed by the pair's MMAs
    uint64_t acc_full[kAccs];     // both: accumulator ready
    uint64_t acc_empty[kAccs];    // leader: both CTAs drained the accumulator
    uint64_t mma_done;
    uint32_t tmem_base;
    alignas(128) float stage[4][32 * 32];  // epilogue: one 32 x 32 fp32 block per epilogue warp
};

enum : unsigned { kSiteEmpty = 0x41, kSiteFull, kSiteAcc, kSiteDone, kSiteAccEmpty };

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA tile load into this CTA's shared memory; completion is counted on the
// mbarrier at `bar_cluster` (the leader's), as a pair member.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
        "%5}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
        : "memory");
}
__device__ __forceinline__ void umma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on the barrier at this offset in both CTAs of the pair once the issued MMAs complete.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
    const uint16_t mask = 0x3;
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(mask)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
gemm_bf16_tn_2sm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        const Params p) {
    pdl_enter();
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int cluster = static_cast<int>(blockIdx.x) >> 1;
    const int nclusters = static_cast<int>(gridDim.x) >> 1;
    const int nk = (p.K + kBK - 1) / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        for (int a = 0; a < kAccs; ++a) {
            mbar_init(&sm.acc_full[a], 1);
            mbar_init(&sm.acc_empty[a], 8);  // 4 epilogue warps x 2 CTAs
        }
        mbar_init(&sm.mma_done, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(&sm.tmem_base, kAccs * kBN);
        tmem_relinquish_pair();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
    }
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised before any cross-CTA arrive
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------
        if (lane == 0) {
            int kit = 0;
            bool ok = true;
            for (int t = cluster; ok && t < p.num_tiles; t += nclusters) {
                if (dt::gemm::tile_is_padding(p, dt::gemm::tile_m(p, t) * kBM)) continue;
                const int m0 = dt::gemm::tile_m(p, t) * kBM + (int)rank * kHalf;
                const int n0 = dt::gemm::tile_n(p, t) * kBN + (int)rank * kHalf;
                for (int kb = 0; kb < nk; ++kb, ++kit) {
                    const int s = kit % kStages;
                    if (!mbar_wait(&sm.empty[s], ((kit / kStages) & 1) ^ 1, kSiteEmpty)) { ok = false; break; }
                    const uint32_t full_leader = peer_addr(&sm.full[s], 0);
                    if (leader) mbar_arrive_expect_tx(&sm.full[s], 2 * (kABytes + kBBytes));
                    if (p.a_plane_k) {
                        const int plane = (kb * kBK) / p.a_plane_k;
                        tma_load_3d_pair(sm.a[s], &tmap_a, full_leader, kb * kBK - plane * p.a_plane_k, m0, plane);
                    } else {
                        tma_load_2d_pair(sm.a[s], &tmap_a, full_leader, kb * kBK, m0);
                    }
                    tma_load_2d_pair(sm.b[s], &tmap_b, full_leader, kb * kBK, n0);
                }
            }
            // before exiting, make sure this CTA's last copies have landed (the
            // leader's full barriers count them; the leader's MMA consumed them)
            if (ok && leader) {
                for (int k = max(0, kit - kStages); k < kit; ++k)
                    mbar_wait(&sm.full[k % kStages], (k / kStages) & 1, kSiteFull);
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer (leader) -----------------
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = umma_idesc_bf16(kBM, kBN, 0, 0);
            int kit = 0, it = 0;
            bool ok = true;
            for (int t = cluster; ok && t < p.num_tiles; t += nclusters) {
                if (dt::gemm::tile_is_padding(p, dt::gemm::tile_m(p, t) * kBM)) continue;
                const int acc = it & 1;
                const uint32_t empty_phase = ((it >> 1) & 1) ^ 1;
                ++it;
                if (!mbar_wait(&sm.acc_empty[acc], empty_phase, kSiteAccEmpty)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d = tmem + acc * kBN;
                for (int kb = 0; kb < nk; ++kb, ++kit) {
                    const int s = kit % kStages;
                    if (!mbar_wait(&sm.full[s], (kit / kStages) & 1, kSiteFull)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sm.a[s]);
                    const uint32_t b0 = smem_u32(sm.b[s]);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        umma_ss_pair(d, umma_desc_sw128(a0 + kk * 32, 16, 1024),
                                     umma_desc_sw128(b0 + kk * 32, 16, 1024), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    umma_commit_pair(&sm.empty[s]);
                }
                if (ok) umma_commit_pair(&sm.acc_full[acc]);
            }
            umma_commit_pair(&sm.mma_done);
            mbar_wait(&sm.mma_done, 0, kSiteDone);
        }
        __syncwarp();
    } else {
        // -------------------------------- epilogue --------------------------
        const int q = warp & 3;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        int it = 0;
        for (int t = cluster; t < p.num_tiles; t += nclusters) {
            const int row = dt::gemm::tile_m(p, t) * kBM + (int)rank * kHalf + q * 32 + lane;
            const int n0 = dt::gemm::tile_n(p, t) * kBN;
            if (dt::gemm::tile_is_padding(p, dt::gemm::tile_m(p, t) * kBM)) {
                if (p.pad_zero && p.epilogue == dt::gemm::kStore) {
                    float z[32];
#pragma unroll
                    for (int e = 0; e < 32; ++e) z[e] = 0.f;
#pragma unroll 1
                    for (int cc = 0; cc < kBN / 32; ++cc) dt::gemm::store_chunk(p, row, n0 + cc * 32, z);
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
            const uint32_t taddr = tmem + lane_off + acc * kBN;
            if (p.epilogue == dt::gemm::kSwiGLU) {
                // Both CTAs hold all 256 columns of their rows: [0,128) gate, [128,256) up.
                const int oc0 = dt::gemm::tile_n(p, t) * (kBN / 2);
#pragma unroll 1
                for (int cc = 0; cc < kBN / 64; ++cc) {
                    float g[32], u[32];
                    tmem_ld32(taddr + cc * 32, g);
                    tmem_ld32(taddr + kBN / 2 + cc * 32, u);
                    tmem_wait_ld();
                    const int oc = oc0 + cc * 32;
                    if (row < p.M && oc + 32 <= p.N / 2) {
                        uint4* dd = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.C) +
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
                            dd[i] = w;
                        }
                    }
                }
            } else {
                const uint32_t stage = smem_u32(sm.stage[q]);
#pragma unroll 1
                for (int cc = 0; cc < kBN / 32; ++cc) {
                    float v[32];
                    tmem_ld32(taddr + cc * 32, v);
                    tmem_wait_ld();
                    if (dt::gemm::staged_f32(p, n0 + cc * 32))
                        dt::gemm::store_rows_f32_staged(p, stage, row - lane, n0 + cc * 32, v, lane);
                    else
                        dt::gemm::store_chunk(p, row, n0 + cc * 32, v);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(peer_addr(&sm.acc_empty[acc], 0));
        }
    }

    tc_fence_before();
    cluster_sync();  // no CTA leaves while its peer may still signal its barriers
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, kAccs * kBN);
    }
}

}  // namespace gemm2
}  // namespace dt
