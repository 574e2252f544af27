// extern "C" layer of the B200 attention hot path (declared in
// include/dirktensor_b200.h).  The whole library is this one translation unit:
// the kernel headers are included below.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <chrono>
#include <cstring>
#include <utility>
#include <mutex>
#include <thread>
#include <string>
#include <vector>

#include "../../include/dirktensor_b200.h"
#include "dt_common.cuh"
#include "flash_bwd.cuh"
#include "flash_fwd.cuh"
#include "gemm.cuh"
#include "gemm2sm.cuh"
#include "model.cuh"
#include "prologue.cuh"

namespace dt {
// Diagnostic for the failure path: one thread waits on an mbarrier that nothing
// arrives on.  mbar_wait gives up after its budget, records the site in the
// device error word and the kernel returns normally.
__global__ void expired_wait_kernel(unsigned site) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        mbar_wait(&bar, 0, site);
    }
}
}  // namespace dt

namespace {

constexpr int kVersion = 100;  // 0.1.0
constexpr int kMaxSeqLen = 8192;  // model_config.h:4 (RoPE table length)

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

#define DT_CUDA(call)                                                                                    \
    do {                                                                                                 \
        cudaError_t e_ = (call);                                                                         \
        if (e_ != cudaSuccess)                                                                           \
            return fail(e_ == cudaErrorMemoryAllocation ? DT_ERR_OUT_OF_MEMORY : DT_ERR_CUDA, "%s: %s (%s:%d)", \
                        #call, cudaGetErrorString(e_), __FILE__, __LINE__);                              \
    } while (0)

#define DT_TRY(expr)              \
    do {                          \
        int s_ = (expr);          \
        if (s_ != DT_OK) return s_; \
    } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// Tensor maps through the driver entry point (no link-time libcuda dependency)
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode(EncodeTiledFn* out) {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    static cudaError_t err = cudaSuccess;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&fn), cudaEnableDefault, &q);
        if (err == cudaSuccess && q != cudaDriverEntryPointSuccess) err = cudaErrorNotSupported;
    });
    if (err != cudaSuccess || fn == nullptr)
        return fail(DT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable: %s", cudaGetErrorString(err));
    *out = fn;
    return DT_OK;
}

// bf16 [B, T, H, D] token-major -> 4-D map (D, H, T, B), box 64 x 1 x 128 x 1, 128 B swizzle.
int make_map_bthd(CUtensorMap* m, const void* base, int B, int T, int H, int D) {
    EncodeTiledFn enc;
    DT_TRY(get_encode(&enc));
    const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)T, (cuuint64_t)B};
    const cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)H * D * 2, (cuuint64_t)T * H * D * 2};
    const cuuint32_t box[4] = {64, 1, 128, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(DT_ERR_CUDA, "cuTensorMapEncodeTiled(BTHD) failed: %d", (int)r);
    return DT_OK;
}

// bf16 row-major [rows, K] -> 2-D map (K, rows), box 64 x box_rows, 128 B swizzle.
int make_map_2d(CUtensorMap* m, const void* base, long long rows, int K, int box_rows) {
    EncodeTiledFn enc;
    DT_TRY(get_encode(&enc));
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(DT_ERR_CUDA, "cuTensorMapEncodeTiled(2D) failed: %d", (int)r);
    return DT_OK;
}

// bf16 planar A: `planes` arrays [rows, plane_k] back to back -> 3-D map
// (plane_k, rows, planes), box 64 x 128 x 1, 128 B swizzle.
int make_map_planar(CUtensorMap* m, const void* base, long long rows, int plane_k, int planes) {
    EncodeTiledFn enc;
    DT_TRY(get_encode(&enc));
    const cuuint64_t dims[3] = {(cuuint64_t)plane_k, (cuuint64_t)rows, (cuuint64_t)planes};
    const cuuint64_t strides[2] = {(cuuint64_t)plane_k * 2, (cuuint64_t)rows * plane_k * 2};
    const cuuint32_t box[3] = {64, (cuuint32_t)dt::gemm::kBM, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(DT_ERR_CUDA, "cuTensorMapEncodeTiled(planar) failed: %d", (int)r);
    return DT_OK;
}

// ---------------------------------------------------------------------------
// Per-device state: kernel attributes, RoPE tables, host-API staging buffers
// ---------------------------------------------------------------------------
struct DevState {
    bool attrs = false;
    int num_sms = 148;
    float* sin_t = nullptr;
    float* cos_t = nullptr;
    float rope_theta = 0.f;
    cudaStream_t stream = nullptr;  // host-buffer entry points
    void* stage = nullptr;
    size_t stage_bytes = 0;
};
std::mutex g_mu;
DevState g_dev[64];

constexpr size_t kFlashSmem = sizeof(dt::attn_fwd::Smem) + 1024;
constexpr size_t kFlashBwdKvSmem = sizeof(dt::attn_bwd::SmemKV) + 1024;
constexpr size_t kFlashBwdQSmem = sizeof(dt::attn_bwd::SmemQ) + 1024;
constexpr size_t kGemmSmem = sizeof(dt::gemm::SmemT<dt::gemm::kBN>) + 1024;
constexpr size_t kGemmNarrowSmem = sizeof(dt::gemm::SmemT<dt::gemm::kNarrowBN>) + 1024;
constexpr size_t kGemm2Smem = sizeof(dt::gemm2::Smem) + 1024;
// GEMMs with at least this many rows run on SM pairs (gemm2sm.cuh); measured on
// B200 at the model's shapes the pair kernel is 18-57 % faster than the one-SM
// kernel, which remains for row counts below one pair tile's half.
// QK-norm/RoPE prologue: 0 = one CTA per token; n > 0 = a persistent grid of n CTAs per SM
// that prefetches each CTA's next token.  Measured on B200 (L2 flushed), 16384 tokens:
// one CTA per token 139-140 us, n = 2 122-123 us (115 registers, no spills), n = 3 (capped
// at 85 registers: spills) 164 us; 131072 tokens 1028 / 871 / 1197 us.
#ifndef DT_PROLOGUE_PERSISTENT
#define DT_PROLOGUE_PERSISTENT 2
#endif
// Attention on grids of fewer 256-row blocks than SMs runs one 128-row Q tile per CTA.
#ifndef DT_FLASH_SMALL_GRID_ONE_TILE
#define DT_FLASH_SMALL_GRID_ONE_TILE 1
#endif
// The pair kernel needs at least this many 256 x 256 tiles per 100 SM pairs.  Measured on
// B200 (CUDA events, L2 flushed): M=512, N=6144, K=2048 (48 pair tiles on 74 pairs) 30.7 us on
// pairs vs 34.9 us on 192 one-SM 128 x 128 tiles; M=N=K=2048 (64 pair tiles) 26.6 vs 34.8 us;
// M=512, N=2048 (16 pair tiles) 24.6 vs 20.5 us on 64 one-SM tiles.
#ifndef DT_GEMM_PAIR_MIN_FILL
#define DT_GEMM_PAIR_MIN_FILL 40
#endif
#ifndef DT_GEMM_2SM_MIN_M
#define DT_GEMM_2SM_MIN_M 256
#endif

// Makes a handle's device current for the scope of an entry point and puts the
// caller's current device back on every return path.
class DeviceGuard {
public:
    int enter(int device) {
        DT_CUDA(cudaGetDevice(&prev_));
        if (prev_ != device) {
            DT_CUDA(cudaSetDevice(device));
            restore_ = true;
        }
        return DT_OK;
    }
    ~DeviceGuard() {
        if (restore_) cudaSetDevice(prev_);
    }

private:
    int prev_ = 0;
    bool restore_ = false;
};

// Programmatic dependent launch (PDL) for the kernels that begin with pdl_enter()
// (the cast, both GEMMs, the prologue and the attention kernel): launched with the
// programmatic-serialization attribute, a kernel's CTAs may be dispatched while the
// previous kernel on the stream finishes; they wait in pdl_enter() until it has
// completed, before any global memory access.  0 launches them plainly.
#ifndef DT_PDL
#define DT_PDL 1
#endif

template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
#if DT_PDL
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    DT_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
#else
    kernel<<<grid, block, smem, st>>>(std::forward<Args>(args)...);
    DT_CUDA(cudaGetLastError());
#endif
    return DT_OK;
}

int current_device(int* dev) {
    DT_CUDA(cudaGetDevice(dev));
    if (*dev < 0 || *dev >= 64) return fail(DT_ERR_UNSUPPORTED, "device index %d out of range", *dev);
    return DT_OK;
}

// Called with g_mu held.
int ensure_attrs(int dev) {
    DevState& s = g_dev[dev];
    if (s.attrs) return DT_OK;
    cudaDeviceProp prop;
    DT_CUDA(cudaGetDeviceProperties(&prop, dev));
    if (prop.major != 10)
        return fail(DT_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a only", dev,
                    prop.major, prop.minor);
    s.num_sms = prop.multiProcessorCount;
    DT_CUDA(cudaFuncSetAttribute(dt::attn_bwd::attn_bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kFlashBwdKvSmem));
    DT_CUDA(cudaFuncSetAttribute(dt::attn_bwd::attn_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kFlashBwdQSmem));
    DT_CUDA(cudaFuncSetAttribute(dt::attn_fwd::attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kFlashSmem));
    DT_CUDA(cudaFuncSetAttribute(dt::gemm::gemm_bf16_tn_kernel<dt::gemm::kBN>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem));
    DT_CUDA(cudaFuncSetAttribute(dt::gemm::gemm_bf16_tn_kernel<dt::gemm::kNarrowBN>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmNarrowSmem));
    DT_CUDA(cudaFuncSetAttribute(dt::gemm2::gemm_bf16_tn_2sm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kGemm2Smem));
    s.attrs = true;
    return DT_OK;
}

int prepare_device(int* dev_out) {
    int dev;
    DT_TRY(current_device(&dev));
    std::lock_guard<std::mutex> lk(g_mu);
    DT_TRY(ensure_attrs(dev));
    *dev_out = dev;
    return DT_OK;
}

void rope_tables_host(std::vector<float>& sin_t, std::vector<float>& cos_t, int max_seq, int head_dim,
                      double theta) {
    // compute_rope_buffers (OlmoAttention.cpp:18-36): inv_freq in double, angle
    // p * inv_freq[j mod half], sin/cos in double, cast to float.
    const int half = head_dim / 2;
    sin_t.resize((size_t)max_seq * head_dim);
    cos_t.resize((size_t)max_seq * head_dim);
    std::vector<double> inv(half);
    for (int i = 0; i < half; ++i) inv[i] = 1.0 / std::pow(theta, (double)(2 * i) / (double)head_dim);
    for (int p = 0; p < max_seq; ++p)
        for (int j = 0; j < head_dim; ++j) {
            const double a = (double)p * inv[j % half];
            sin_t[(size_t)p * head_dim + j] = (float)std::sin(a);
            cos_t[(size_t)p * head_dim + j] = (float)std::cos(a);
        }
}

int ensure_rope(int dev, float theta, const float** sin_t, const float** cos_t) {
    std::lock_guard<std::mutex> lk(g_mu);
    DevState& s = g_dev[dev];
    if (s.sin_t == nullptr || s.rope_theta != theta) {
        std::vector<float> hs, hc;
        rope_tables_host(hs, hc, kMaxSeqLen, 128, (double)theta);
        const size_t bytes = hs.size() * sizeof(float);
        if (s.sin_t == nullptr) {
            DT_CUDA(cudaMalloc(&s.sin_t, bytes));
            DT_CUDA(cudaMalloc(&s.cos_t, bytes));
        }
        DT_CUDA(cudaMemcpy(s.sin_t, hs.data(), bytes, cudaMemcpyHostToDevice));
        DT_CUDA(cudaMemcpy(s.cos_t, hc.data(), bytes, cudaMemcpyHostToDevice));
        s.rope_theta = theta;
    }
    *sin_t = s.sin_t;
    *cos_t = s.cos_t;
    return DT_OK;
}

// Host-API staging buffer of at least `bytes` on `dev` (called with g_mu held).
int ensure_stage(int dev, size_t bytes, void** out, cudaStream_t* stream) {
    DevState& s = g_dev[dev];
    if (s.stream == nullptr) DT_CUDA(cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking));
    if (s.stage_bytes < bytes) {
        if (s.stage) DT_CUDA(cudaFree(s.stage));
        s.stage = nullptr;
        s.stage_bytes = 0;
        DT_CUDA(cudaMalloc(&s.stage, bytes));
        s.stage_bytes = bytes;
    }
    *out = s.stage;
    *stream = s.stream;
    return DT_OK;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
int launch_cast(const float* src, void* dst, long long n, cudaStream_t st) {
    if (n == 0) return DT_OK;
    const long long n4 = n / 4;
    const int threads = 256;
    long long blocks = (n4 + threads - 1) / threads;
    if (blocks > 148 * 16) blocks = 148 * 16;
    return launch_pdl(dt::elem::cast_f32_bf16_kernel, dim3((unsigned)blocks), dim3(threads), 0, st,
                      reinterpret_cast<const float4*>(src), reinterpret_cast<uint2*>(dst), n4);
}

// Casts the first `count` (1..3) of a, b, c in one launch.
int launch_cast3(const float* a, const float* b, const float* c, void* da, void* db, void* dc, long long n,
                 cudaStream_t st, int count = 3) {
    if (n == 0) return DT_OK;
    dt::elem::Cast3 args;
    args.src[0] = reinterpret_cast<const float4*>(a);
    args.src[1] = reinterpret_cast<const float4*>(b);
    args.src[2] = reinterpret_cast<const float4*>(c);
    args.dst[0] = reinterpret_cast<uint2*>(da);
    args.dst[1] = reinterpret_cast<uint2*>(db);
    args.dst[2] = reinterpret_cast<uint2*>(dc);
    const long long n4 = n / 4;
    const int threads = 256;
    long long blocks = (n4 + threads - 1) / threads;
    if (blocks > 148 * 8) blocks = 148 * 8;
    dt::elem::cast3_f32_bf16_kernel<<<dim3((unsigned)blocks, (unsigned)count), threads, 0, st>>>(args, n4);
    DT_CUDA(cudaGetLastError());
    return DT_OK;
}

struct Scatter {
    int ranks = 0;
    int plane = 0;
    long long tokens_per_rank = 0;
    void* const* dst = nullptr;
};

// q: bf16 [B, T, H, D] read through a tensor map, or, when q_f32 is given, unused
// (the kernel reads the fp32 rows itself; the K map stands in for the Q map).
int launch_flash(const void* q, const void* k, const void* v, void* o, int o_bf16, long long o_row_stride,
                 float* m, float* l, const int* seq_lens, int B, int T, int H, float scale, int causal,
                 cudaStream_t st, const Scatter& sc = Scatter(), const float* q_f32 = nullptr) {
    if ((long long)B * T * H == 0) return DT_OK;
    CUtensorMap mq, mk, mv;
    DT_TRY(make_map_bthd(&mq, q_f32 ? k : q, B, T, H, 128));
    DT_TRY(make_map_bthd(&mk, k, B, T, H, 128));
    DT_TRY(make_map_bthd(&mv, v, B, T, H, 128));
    dt::attn_fwd::Params p{};
    p.B = B;
    p.T = T;
    p.H = H;
    {
        int dev = 0;
        cudaGetDevice(&dev);
        const int sms = (dev >= 0 && dev < 64) ? g_dev[dev].num_sms : 148;
        const int BH = B * H;
        // One Q tile per CTA (128-row work items) when 256-row blocks would not
        // give every SM a CTA (short sequences, few heads): twice the CTAs, each
        // half as long.
        p.qtiles = (DT_FLASH_SMALL_GRID_ONE_TILE && (long long)BH * ((T + 255) / 256) < sms) ? 1 : 2;
        p.nblk = (T + 128 * p.qtiles - 1) / (128 * p.qtiles);
        // Scheduling groups of (b, h) pairs.  When the K/V of all heads fit in L2
        // (<= 64 MB of bf16) one group keeps a global heaviest-first order.
        // Otherwise each group holds about two waves of blocks -- enough to fill
        // the GPU, few enough heads that their K/V stay in L2 -- and the groups
        // are sized evenly so the last one is not a short tail.
        const double kv_bytes = (double)BH * T * 128 * 2 * 2;
        if (kv_bytes <= 64.0 * 1024 * 1024) {
            p.group = BH;
        } else {
            const int want = std::max(1, (2 * sms + p.nblk - 1) / p.nblk);
            const int ngroups = (BH + want - 1) / want;
            p.group = (BH + ngroups - 1) / ngroups;
        }
    }
    p.causal = causal ? 1 : 0;
    p.scale = scale;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.out = o;
    p.out_bf16 = o_bf16;
    p.out_row_stride = o_row_stride;
    p.m_out = m;
    p.l_out = l;
    p.seq_lens = seq_lens;
    p.scatter_ranks = sc.ranks;
    p.scatter_plane = sc.plane;
    p.tokens_per_rank = sc.tokens_per_rank;
    for (int r = 0; r < 8; ++r) p.scatter_dst[r] = (r < sc.ranks) ? sc.dst[r] : nullptr;
    p.q_f32 = q_f32;
    p.q_row_stride = (long long)H * 128;
    const long long grid = (long long)p.nblk * B * H;
    if (grid > 0x7fffffffLL) return fail(DT_ERR_INVALID_ARGUMENT, "problem too large (%lld CTAs)", grid);
    return launch_pdl(dt::attn_fwd::attn_fwd_kernel, dim3((unsigned)grid), dim3(dt::attn_fwd::kThreads), kFlashSmem, st,
                      mq, mk, mv, p);
}

// Attention backward on bf16 Q/K/V.  dout fp32 [B,T,H,D]; O fp32 (out) or bf16
// (out_bf16) with row stride out_row_stride; m, l [B,T,H]; dq/dk/dv fp32
// [B,T,H,D].  Scratch: dob (bf16 [B,T,H,D]), dvec and lse2 ([B,H,Tpad] fp32).
size_t flash_bwd_rows_bytes(int B, int T, int H) {
    const long long Tpad = (long long)((T + 127) / 128) * 128;
    return align256((size_t)B * H * Tpad * 4);
}

int launch_flash_bwd(const void* qb, const void* kb, const void* vb, const float* dout, const float* out,
                     const void* out_bf16, long long out_row_stride, const float* m, const float* l, float* dq,
                     float* dk, float* dv, int B, int T, int H, float scale, int causal, void* dob, float* dvec,
                     float* lse2, cudaStream_t st) {
    if ((long long)B * T * H == 0) return DT_OK;
    const int nblk = (T + 127) / 128;
    dt::attn_bwd::PreParams pp{};
    pp.out = out;
    pp.out_bf16 = reinterpret_cast<const __nv_bfloat16*>(out_bf16);
    pp.out_row_stride = out_row_stride;
    pp.dout = dout;
    pp.m = m;
    pp.l = l;
    pp.dout_bf16 = reinterpret_cast<__nv_bfloat16*>(dob);
    pp.dvec = dvec;
    pp.lse2 = lse2;
    pp.B = B;
    pp.T = T;
    pp.H = H;
    pp.Tpad = nblk * 128;
    const long long rows = (long long)B * H * pp.Tpad;
    dt::attn_bwd::attn_bwd_pre_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(pp);
    DT_CUDA(cudaGetLastError());
    CUtensorMap mq, mk, mv, mdo;
    DT_TRY(make_map_bthd(&mq, qb, B, T, H, 128));
    DT_TRY(make_map_bthd(&mk, kb, B, T, H, 128));
    DT_TRY(make_map_bthd(&mv, vb, B, T, H, 128));
    DT_TRY(make_map_bthd(&mdo, dob, B, T, H, 128));
    dt::attn_bwd::Params p{};
    p.B = B;
    p.T = T;
    p.H = H;
    p.nblk = nblk;
    p.Tpad = pp.Tpad;
    p.causal = causal ? 1 : 0;
    p.scale = scale;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.dvec = dvec;
    p.lse2 = lse2;
    p.dq = dq;
    p.dk = dk;
    p.dv = dv;
    const long long grid = (long long)nblk * B * H;
    if (grid > 0x7fffffffLL) return fail(DT_ERR_INVALID_ARGUMENT, "problem too large (%lld CTAs)", grid);
    dt::attn_bwd::attn_bwd_dkdv_kernel<<<(unsigned)grid, dt::attn_bwd::kThreads, kFlashBwdKvSmem, st>>>(
        mq, mk, mv, mdo, p);
    DT_CUDA(cudaGetLastError());
    dt::attn_bwd::attn_bwd_dq_kernel<<<(unsigned)grid, dt::attn_bwd::kThreads, kFlashBwdQSmem, st>>>(mq, mk, mv,
                                                                                                      mdo, p);
    DT_CUDA(cudaGetLastError());
    return DT_OK;
}

// seq_lens/seq_T (optional): right-padded batch; output tiles entirely in a
// sequence's padding are skipped (and written as zeros when pad_zero).
// split_c2 / split_ldc2 / split_col0: columns >= split_col0 go to split_c2 as bf16 (kStore only).
int launch_gemm(const void* A, const void* Bm, void* C, int c_bf16, int M, int N, int K, long long ldc,
                cudaStream_t st, int a_planes = 1, int epilogue = dt::gemm::kStore, const int* seq_lens = nullptr,
                int seq_T = 0, int pad_zero = 0, int a_mn = 0, int b_mn = 0, void* split_c2 = nullptr,
                long long split_ldc2 = 0, int split_col0 = 0) {
    if (M == 0 || N == 0) return DT_OK;
    CUtensorMap ma, mb;
    const int plane_k = K / a_planes;
    int dev0 = 0;
    cudaGetDevice(&dev0);
    const int nsm = (dev0 >= 0 && dev0 < 64) ? g_dev[dev0].num_sms : 148;
    // Tile choice: 256 x 256 tiles on SM pairs when they fill at least every
    // pair; otherwise 128 x 256 tiles on single SMs, narrowed to 128 x 128 when
    // the wide tiles would leave SMs idle (the SwiGLU epilogue needs 256 columns).
    const long long pair_tiles = (long long)((M + 255) / 256) * ((N + 255) / 256);
    const long long wide_tiles = (long long)((M + 127) / 128) * ((N + 255) / 256);
    // (MN-major operands run on the one-SM kernel)
    const bool pair = M >= DT_GEMM_2SM_MIN_M && N >= 256 && pair_tiles * 100 >= (long long)(nsm / 2) * DT_GEMM_PAIR_MIN_FILL &&
                      !a_mn && !b_mn;
    const bool narrow = !pair && epilogue != dt::gemm::kSwiGLU && wide_tiles < nsm;
    const int bn = narrow ? dt::gemm::kNarrowBN : dt::gemm::kBN;
    // boxes: 128 rows of A and bn rows of B per CTA, or 128 and 128 on SM pairs
    // MN-major operands ([K, M] / [K, N] row-major): 64 x 64 boxes
    if (a_mn) DT_TRY(make_map_2d(&ma, A, K, M, 64));
    else if (a_planes > 1) DT_TRY(make_map_planar(&ma, A, M, plane_k, a_planes));
    else DT_TRY(make_map_2d(&ma, A, M, K, dt::gemm::kBM));
    if (b_mn) DT_TRY(make_map_2d(&mb, Bm, K, N, 64));
    else DT_TRY(make_map_2d(&mb, Bm, N, K, pair ? dt::gemm2::kHalf : bn));
    dt::gemm::Params p{};
    p.M = M;
    p.N = N;
    p.K = K;
    p.C = C;
    p.ldc = ldc;
    p.c_bf16 = c_bf16;
    p.a_plane_k = a_planes > 1 ? plane_k : 0;
    p.epilogue = epilogue;
    p.a_mn = a_mn;
    p.b_mn = b_mn;
    if (split_c2) {
        if (epilogue != dt::gemm::kStore || c_bf16 || (split_col0 % 32) != 0)
            return fail(DT_ERR_INVALID_ARGUMENT, "split output needs an fp32 store epilogue and a column multiple of 32");
        p.C2 = split_c2;
        p.ldc2 = split_ldc2;
        p.c2_col0 = split_col0;
    }
    // tiles are 256 rows on SM pairs, 128 on one SM: skip only if they never straddle sequences
    const int tile_rows = pair ? dt::gemm2::kBM : dt::gemm::kBM;
    if (seq_lens && seq_T > 0 && (seq_T % tile_rows) == 0) {
        p.seq_lens = seq_lens;
        p.seq_T = seq_T;
        p.pad_zero = pad_zero;
    }
    p.tiles_n = (N + bn - 1) / bn;
    p.tiles_m = (M + dt::gemm::kBM - 1) / dt::gemm::kBM;
    p.m_fastest = N > M ? 1 : 0;
    const long long tiles = (long long)p.tiles_n * p.tiles_m;
    if (tiles > 0x7fffffffLL) return fail(DT_ERR_INVALID_ARGUMENT, "GEMM too large");
    p.num_tiles = (int)tiles;
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = (dev >= 0 && dev < 64) ? g_dev[dev].num_sms : 148;
    if (pair) {
        // cluster tiles of 256 x 256 on SM pairs; persistent: one CTA per SM
        p.tiles_n = (N + dt::gemm2::kBN - 1) / dt::gemm2::kBN;
        p.tiles_m = (M + dt::gemm2::kBM - 1) / dt::gemm2::kBM;
        p.num_tiles = p.tiles_n * p.tiles_m;
        const int clusters = std::max(1, std::min(p.num_tiles, sms / 2));
        return launch_pdl(dt::gemm2::gemm_bf16_tn_2sm_kernel, dim3(2 * clusters), dim3(dt::gemm2::kThreads),
                          kGemm2Smem, st, ma, mb, p);
    }
    const int grid = (int)std::min<long long>(tiles, sms);  // persistent: one CTA per SM
    if (narrow)
        return launch_pdl(dt::gemm::gemm_bf16_tn_kernel<dt::gemm::kNarrowBN>, dim3(grid), dim3(dt::gemm::kThreads),
                          kGemmNarrowSmem, st, ma, mb, p);
    return launch_pdl(dt::gemm::gemm_bf16_tn_kernel<dt::gemm::kBN>, dim3(grid), dim3(dt::gemm::kThreads), kGemmSmem,
                      st, ma, mb, p);
}

int launch_prologue(const float* q, const float* k, const float* v, long long ld_in, const float* qg,
                    const float* kg, const float* sin_t, const float* cos_t, void* qo, void* ko, void* vo, int B,
                    int T, float eps, cudaStream_t st) {
    const long long M = (long long)B * T;
    if (M == 0) return DT_OK;
    dt::elem::PrologueParams p;
    p.q = q;
    p.k = k;
    p.v = v;
    p.ld_in = ld_in;
    p.q_gain = qg;
    p.k_gain = kg;
    p.sin_t = sin_t;
    p.cos_t = cos_t;
    p.qo = reinterpret_cast<__nv_bfloat16*>(qo);
    p.ko = reinterpret_cast<__nv_bfloat16*>(ko);
    p.vo = reinterpret_cast<__nv_bfloat16*>(vo);
    p.T = T;
    p.eps = eps;
    if (M > 0x7fffffffLL) return fail(DT_ERR_INVALID_ARGUMENT, "too many rows");
#if DT_PROLOGUE_PERSISTENT
    {
        int dev = 0;
        cudaGetDevice(&dev);
        const int sms = (dev >= 0 && dev < 64) ? g_dev[dev].num_sms : 148;
        const long long grid = std::min<long long>(M, (long long)sms * DT_PROLOGUE_PERSISTENT);
        return launch_pdl(dt::elem::qk_norm_rope_loop_kernel, dim3((unsigned)grid), dim3(dt::elem::kPrologueThreads), 0,
                          st, p, M);
    }
#else
    return launch_pdl(dt::elem::qk_norm_rope_kernel, dim3((unsigned)M), dim3(dt::elem::kPrologueThreads), 0, st, p);
#endif
}

int launch_sumsq(const float* q, const float* k, long long ld, int width, long long M, float* ss, cudaStream_t st) {
    if (M == 0) return DT_OK;
    const long long blocks = (M + 7) / 8;
    if (blocks > 0x7fffffffLL) return fail(DT_ERR_INVALID_ARGUMENT, "too many rows");
    dt::elem::qk_sumsq_kernel<<<(unsigned)blocks, 256, 0, st>>>(q, k, ld, width, M, reinterpret_cast<float2*>(ss));
    DT_CUDA(cudaGetLastError());
    return DT_OK;
}

int launch_prologue_shard(const float* q, const float* k, const float* v, long long ld_in, const float* ss,
                          const float* qg, const float* kg, int heads, const float* sin_t, const float* cos_t,
                          void* qo, void* ko, void* vo, int B, int T, float eps, cudaStream_t st) {
    const long long M = (long long)B * T;
    if (M == 0) return DT_OK;
    dt::elem::ShardPrologueParams p;
    p.q = q;
    p.k = k;
    p.v = v;
    p.ld_in = ld_in;
    p.ss = reinterpret_cast<const float2*>(ss);
    p.q_gain = qg;
    p.k_gain = kg;
    p.sin_t = sin_t;
    p.cos_t = cos_t;
    p.qo = reinterpret_cast<__nv_bfloat16*>(qo);
    p.ko = reinterpret_cast<__nv_bfloat16*>(ko);
    p.vo = reinterpret_cast<__nv_bfloat16*>(vo);
    p.heads = heads;
    p.T = T;
    p.M = M;
    p.eps = eps;
    const int per_cta = dt::elem::kPrologueThreads / (heads * 16);
    const long long blocks = (M + per_cta - 1) / per_cta;
    if (blocks > 0x7fffffffLL) return fail(DT_ERR_INVALID_ARGUMENT, "too many rows");
    dt::elem::qk_norm_rope_shard_kernel<<<(unsigned)blocks, dt::elem::kPrologueThreads, 0, st>>>(p);
    DT_CUDA(cudaGetLastError());
    return DT_OK;
}

int check_flash_shape(int B, int T, int H, int D) {
    if (B < 0 || T < 0 || H < 0) return fail(DT_ERR_INVALID_ARGUMENT, "negative shape B=%d T=%d H=%d", B, T, H);
    if (D != 128) return fail(DT_ERR_UNSUPPORTED, "head_dim %d unsupported (must be 128)", D);
    return DT_OK;
}

int read_device_error(bool* had) {
    unsigned code = 0, info = 0;
    DT_CUDA(cudaMemcpyFromSymbol(&code, dt::g_dev_error, sizeof(code)));
    *had = code != 0;
    if (code) {
        DT_CUDA(cudaMemcpyFromSymbol(&info, dt::g_dev_error_info, sizeof(info)));
        const unsigned zero = 0;
        DT_CUDA(cudaMemcpyToSymbol(dt::g_dev_error, &zero, sizeof(zero)));
        return fail(DT_ERR_DEVICE_TIMEOUT, "a kernel wait expired (site 0x%x, parity %u); results are invalid",
                    code & 0xffu, info);
    }
    return DT_OK;
}

}  // namespace

// ===========================================================================
// NCCL, loaded at run time (the single-GPU entry points need no NCCL)
// ===========================================================================
namespace {
struct NcclApi {
    bool loaded = false;
    std::string err;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi& nccl_api() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char* e = dlerror();
            api.err = e ? e : "dlopen(libnccl.so.2) failed";
            return;
        }
#define DT_NCCL_SYM(field, sym)                                              \
    api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, sym));        \
    if (!api.field) {                                                        \
        api.err = std::string("libnccl.so.2 has no ") + sym;                 \
        return;                                                              \
    }
        DT_NCCL_SYM(GetUniqueId, "ncclGetUniqueId")
        DT_NCCL_SYM(CommInitRankConfig, "ncclCommInitRankConfig")
        DT_NCCL_SYM(CommGetAsyncError, "ncclCommGetAsyncError")
        DT_NCCL_SYM(CommAbort, "ncclCommAbort")
        DT_NCCL_SYM(CommDestroy, "ncclCommDestroy")
        DT_NCCL_SYM(AllReduce, "ncclAllReduce")
        DT_NCCL_SYM(AllGather, "ncclAllGather")
        DT_NCCL_SYM(Send, "ncclSend")
        DT_NCCL_SYM(Recv, "ncclRecv")
        DT_NCCL_SYM(GroupStart, "ncclGroupStart")
        DT_NCCL_SYM(GroupEnd, "ncclGroupEnd")
        DT_NCCL_SYM(GetErrorString, "ncclGetErrorString")
#undef DT_NCCL_SYM
        api.loaded = true;
    });
    return api;
}

int need_nccl(NcclApi** out) {
    NcclApi& n = nccl_api();
    if (!n.loaded) return fail(DT_ERR_NCCL, "NCCL unavailable: %s", n.err.c_str());
    *out = &n;
    return DT_OK;
}
}  // namespace

struct dt_comm {
    ncclComm_t comm = nullptr;
    int world = 1, rank = 0, device = 0;
    int timeout_ms = 60000;
};

namespace {
// The communicator is non-blocking: a call may return ncclInProgress while
// NCCL finishes it in the background.  Polls until it is done, giving up
// (and aborting the communicator) after the communicator's timeout.
int nccl_done(dt_comm* c, ncclResult_t r, const char* what) {
    NcclApi& n = nccl_api();
    if (r == ncclInProgress) {
        const auto t0 = std::chrono::steady_clock::now();
        for (;;) {
            ncclResult_t st = ncclSuccess;
            const ncclResult_t q = n.CommGetAsyncError(c->comm, &st);
            if (q != ncclSuccess) {
                r = q;
                break;
            }
            if (st != ncclInProgress) {
                r = st;
                break;
            }
            const auto us =
                std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0).count();
            if (us > 1000LL * c->timeout_ms) {
                n.CommAbort(c->comm);
                c->comm = nullptr;
                return fail(DT_ERR_TIMEOUT, "%s did not complete within %d ms; the communicator was aborted", what,
                            c->timeout_ms);
            }
            // An enqueue finishes within microseconds: spin first (the GPU may be
            // idle until the next launch is queued), sleep only for long waits
            // (communicator set-up).
            if (us < 2000) std::this_thread::yield();
            else std::this_thread::sleep_for(std::chrono::microseconds(100));
        }
    }
    if (r != ncclSuccess) return fail(DT_ERR_NCCL, "%s: %s", what, n.GetErrorString(r));
    return DT_OK;
}

int comm_ok(dt_comm* c) {
    if (!c || !c->comm) return fail(DT_ERR_INVALID_ARGUMENT, "communicator is null or was aborted");
    return DT_OK;
}

// State of a head-sharded attention handle (dt_attn_create_sharded).
struct ShardState {
    dt_comm* comm = nullptr;
    int exchange = 0;  // 0: attention kernel stores into the owners' buffers (IPC), 1: NCCL all-to-all
    int h0 = 0, heads = 16;
    // exchange 0: two receive buffers [G, M/G, w] bf16 (one per step parity) and the
    // barrier's flag array (8 counters), and every rank's mapping of all three;
    // rebuilt when M changes
    long long recv_tokens = 0;
    void* recv[3] = {nullptr, nullptr, nullptr};
    void* peers[3][8] = {};
    bool opened[3][8] = {};
    unsigned step = 0;
};
}  // namespace

// ===========================================================================
// extern "C"
// ===========================================================================
struct dt_attn {
    int device = 0;
    int d_model = 0, n_heads = 0;
    float eps = 1e-6f, theta = 500000.f;
    __nv_bfloat16* wqkv = nullptr;  // [3*d, d]
    __nv_bfloat16* wo = nullptr;    // [d, d]
    float* qg = nullptr;
    float* kg = nullptr;
    void* ws = nullptr;
    size_t ws_bytes = 0;
    void* io = nullptr;  // host-API staging: x, y, seq_lens
    size_t io_bytes = 0;
    cudaStream_t stream = nullptr;
    // training path (OlmoAttention::backward / step / zero_grad)
    float* master = nullptr;  // fp32 weights [Wq; Wk; Wv] [3d, d] then Wo [d, d] (the bf16 copies derive from these)
    float* grad = nullptr;    // fp32 gradients: [3d, d] | [d, d] | q_norm [d] | k_norm [d]
    void* bws = nullptr;      // backward scratch
    size_t bws_bytes = 0;
    int last_B = 0, last_T = 0;  // shape of the last forward, whose activations the workspace holds
    bool last_varlen = false;
    ShardState* shard = nullptr;  // head-sharded handle (dt_attn_create_sharded)
};

extern "C" {

const char* dt_last_error(void) { return t_last_error.c_str(); }

int dt_version(void) { return kVersion; }

int dt_selftest_expired_wait(void) {
    t_last_error.clear();
    int dev;
    DT_TRY(prepare_device(&dev));
    DT_CUDA(cudaDeviceSynchronize());
    bool had = false;
    DT_TRY(read_device_error(&had));  // start from a clear word
    dt::expired_wait_kernel<<<1, 32>>>(0x7e);
    DT_CUDA(cudaGetLastError());
    DT_CUDA(cudaDeviceSynchronize());
    const int st = read_device_error(&had);
    if (st == DT_ERR_DEVICE_TIMEOUT && had) {
        t_last_error.clear();
        return DT_OK;
    }
    return fail(DT_ERR_CUDA, "expected the wait to expire and be reported (status %d)", st);
}

int dt_check_device_error(void) {
    DT_CUDA(cudaDeviceSynchronize());
    bool had;
    return read_device_error(&had);
}

size_t dt_flash_fwd_workspace_bytes(int B, int T, int H, int D) {
    if (B <= 0 || T <= 0 || H <= 0 || D <= 0) return 0;
    return 3 * align256((size_t)B * T * H * D * 2);
}

int dt_flash_fwd(const float* q, const float* k, const float* v, float* o, float* softmax_m, float* softmax_l,
                 int B, int T, int H, int D, float scale, int causal, void* workspace, size_t workspace_bytes,
                 void* stream) {
    t_last_error.clear();
    DT_TRY(check_flash_shape(B, T, H, D));
    if ((long long)B * T * H == 0) return DT_OK;
    if (!q || !k || !v || !o) return fail(DT_ERR_INVALID_ARGUMENT, "null q/k/v/o");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
        return fail(DT_ERR_INVALID_ARGUMENT, "q/k/v/o must be 16-byte aligned");
    const size_t need = dt_flash_fwd_workspace_bytes(B, T, H, D);
    if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
        return fail(DT_ERR_INVALID_ARGUMENT, "workspace must be >= %zu bytes and 16-byte aligned", need);
    int dev;
    DT_TRY(prepare_device(&dev));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const long long n = (long long)B * T * H * D;
    uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
    const size_t one = align256((size_t)n * 2);
    // K and V to bf16; the attention kernel reads the fp32 Q rows itself
    DT_TRY(launch_cast3(k, v, nullptr, ws + one, ws + 2 * one, nullptr, n, st, 2));
    return launch_flash(nullptr, ws + one, ws + 2 * one, o, 0, (long long)H * D, softmax_m, softmax_l, nullptr, B, T,
                        H, scale, causal, st, Scatter(), q);
}

int dt_flash_fwd_host(const float* q, const float* k, const float* v, float* o, float* softmax_m,
                      float* softmax_l, int B, int T, int H, int D, float scale, int causal) {
    t_last_error.clear();
    DT_TRY(check_flash_shape(B, T, H, D));
    if ((long long)B * T * H == 0) return DT_OK;
    if (!q || !k || !v || !o) return fail(DT_ERR_INVALID_ARGUMENT, "null q/k/v/o");
    int dev;
    DT_TRY(prepare_device(&dev));
    const size_t n = (size_t)B * T * H * D;
    const size_t ns = (size_t)B * T * H;
    const size_t t_bytes = align256(n * 4), s_bytes = align256(ns * 4);
    const size_t ws = dt_flash_fwd_workspace_bytes(B, T, H, D);
    std::lock_guard<std::mutex> lk(g_mu);
    void* stage;
    cudaStream_t st;
    DT_TRY(ensure_stage(dev, 4 * t_bytes + 2 * s_bytes + ws, &stage, &st));
    uint8_t* base = reinterpret_cast<uint8_t*>(stage);
    float* dq = reinterpret_cast<float*>(base);
    float* dk = reinterpret_cast<float*>(base + t_bytes);
    float* dv = reinterpret_cast<float*>(base + 2 * t_bytes);
    float* dout = reinterpret_cast<float*>(base + 3 * t_bytes);
    float* dm = reinterpret_cast<float*>(base + 4 * t_bytes);
    float* dl = reinterpret_cast<float*>(base + 4 * t_bytes + s_bytes);
    void* dws = base + 4 * t_bytes + 2 * s_bytes;
    DT_CUDA(cudaMemcpyAsync(dq, q, n * 4, cudaMemcpyHostToDevice, st));
    DT_CUDA(cudaMemcpyAsync(dk, k, n * 4, cudaMemcpyHostToDevice, st));
    DT_CUDA(cudaMemcpyAsync(dv, v, n * 4, cudaMemcpyHostToDevice, st));
    const long long nn = (long long)n;
    uint8_t* w = reinterpret_cast<uint8_t*>(dws);
    const size_t one = align256(n * 2);
    DT_TRY(launch_cast3(dk, dv, nullptr, w + one, w + 2 * one, nullptr, nn, st, 2));
    DT_TRY(launch_flash(nullptr, w + one, w + 2 * one, dout, 0, (long long)H * D, dm, dl, nullptr, B, T, H, scale,
                        causal, st, Scatter(), dq));
    DT_CUDA(cudaMemcpyAsync(o, dout, n * 4, cudaMemcpyDeviceToHost, st));
    if (softmax_m) DT_CUDA(cudaMemcpyAsync(softmax_m, dm, ns * 4, cudaMemcpyDeviceToHost, st));
    if (softmax_l) DT_CUDA(cudaMemcpyAsync(softmax_l, dl, ns * 4, cudaMemcpyDeviceToHost, st));
    DT_CUDA(cudaStreamSynchronize(st));
    bool had;
    return read_device_error(&had);
}

// ---- flash attention backward ---------------------------------------------

size_t dt_flash_bwd_workspace_bytes(int B, int T, int H, int D) {
    if (B <= 0 || T <= 0 || H <= 0 || D <= 0) return 0;
    return 4 * align256((size_t)B * T * H * D * 2) + 2 * flash_bwd_rows_bytes(B, T, H);
}

int dt_flash_bwd(const float* dout, const float* out, const float* softmax_m, const float* softmax_l,
                 const float* q, const float* k, const float* v, float* dq, float* dk, float* dv, int B, int T,
                 int H, int D, float scale, int causal, void* workspace, size_t workspace_bytes, void* stream) {
    t_last_error.clear();
    DT_TRY(check_flash_shape(B, T, H, D));
    if ((long long)B * T * H == 0) return DT_OK;
    const void* ptrs[] = {dout, out, softmax_m, softmax_l, q, k, v, dq, dk, dv};
    for (const void* ptr : ptrs)
        if (!ptr || !aligned16(ptr)) return fail(DT_ERR_INVALID_ARGUMENT, "null or unaligned (16 B) argument");
    const size_t need = dt_flash_bwd_workspace_bytes(B, T, H, D);
    if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
        return fail(DT_ERR_INVALID_ARGUMENT, "workspace must be >= %zu bytes and 16-byte aligned", need);
    int dev;
    DT_TRY(prepare_device(&dev));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const long long n = (long long)B * T * H * D;
    uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
    const size_t one = align256((size_t)n * 2), rows = flash_bwd_rows_bytes(B, T, H);
    DT_TRY(launch_cast3(q, k, v, ws, ws + one, ws + 2 * one, n, st));
    return launch_flash_bwd(ws, ws + one, ws + 2 * one, dout, out, nullptr, (long long)H * D, softmax_m, softmax_l,
                            dq, dk, dv, B, T, H, scale, causal, ws + 3 * one,
                            reinterpret_cast<float*>(ws + 4 * one), reinterpret_cast<float*>(ws + 4 * one + rows),
                            st);
}

int dt_flash_bwd_host(const float* dout, const float* out, const float* softmax_m, const float* softmax_l,
                      const float* q, const float* k, const float* v, float* dq, float* dk, float* dv, int B, int T,
                      int H, int D, float scale, int causal) {
    t_last_error.clear();
    DT_TRY(check_flash_shape(B, T, H, D));
    if ((long long)B * T * H == 0) return DT_OK;
    const void* ptrs[] = {dout, out, softmax_m, softmax_l, q, k, v, dq, dk, dv};
    for (const void* ptr : ptrs)
        if (!ptr) return fail(DT_ERR_INVALID_ARGUMENT, "null argument");
    int dev;
    DT_TRY(prepare_device(&dev));
    const size_t n = (size_t)B * T * H * D, ns = (size_t)B * T * H;
    const size_t t_bytes = align256(n * 4), s_bytes = align256(ns * 4);
    const size_t ws = dt_flash_bwd_workspace_bytes(B, T, H, D);
    std::lock_guard<std::mutex> lk(g_mu);
    void* stage;
    cudaStream_t st;
    // device copies: dout, out, q, k, v (in), dq, dk, dv (out), m, l, then the workspace
    DT_TRY(ensure_stage(dev, 8 * t_bytes + 2 * s_bytes + ws, &stage, &st));
    uint8_t* base = reinterpret_cast<uint8_t*>(stage);
    float* d[8];
    for (int i = 0; i < 8; ++i) d[i] = reinterpret_cast<float*>(base + i * t_bytes);
    float* dm = reinterpret_cast<float*>(base + 8 * t_bytes);
    float* dl = reinterpret_cast<float*>(base + 8 * t_bytes + s_bytes);
    uint8_t* w = base + 8 * t_bytes + 2 * s_bytes;
    const float* hin[5] = {dout, out, q, k, v};
    for (int i = 0; i < 5; ++i) DT_CUDA(cudaMemcpyAsync(d[i], hin[i], n * 4, cudaMemcpyHostToDevice, st));
    DT_CUDA(cudaMemcpyAsync(dm, softmax_m, ns * 4, cudaMemcpyHostToDevice, st));
    DT_CUDA(cudaMemcpyAsync(dl, softmax_l, ns * 4, cudaMemcpyHostToDevice, st));
    const size_t one = align256(n * 2), rows = flash_bwd_rows_bytes(B, T, H);
    DT_TRY(launch_cast3(d[2], d[3], d[4], w, w + one, w + 2 * one, (long long)n, st));
    DT_TRY(launch_flash_bwd(w, w + one, w + 2 * one, d[0], d[1], nullptr, (long long)H * D, dm, dl, d[5], d[6], d[7],
                            B, T, H, scale, causal, w + 3 * one, reinterpret_cast<float*>(w + 4 * one),
                            reinterpret_cast<float*>(w + 4 * one + rows), st));
    DT_CUDA(cudaMemcpyAsync(dq, d[5], n * 4, cudaMemcpyDeviceToHost, st));
    DT_CUDA(cudaMemcpyAsync(dk, d[6], n * 4, cudaMemcpyDeviceToHost, st));
    DT_CUDA(cudaMemcpyAsync(dv, d[7], n * 4, cudaMemcpyDeviceToHost, st));
    DT_CUDA(cudaStreamSynchronize(st));
    bool had;
    return read_device_error(&had);
}

// ---- flash attention forward without any allocation ------------------------
//
// For callers that must not allocate device memory themselves or have the
// library do it: a serving engine that reserves its whole HBM budget up front
// and hands out every byte through its own pool, a plugin running inside a
// host framework that forbids allocation from its callbacks, or a latency
// critical loop where cudaMalloc/cudaFree (which can synchronise the device)
// are not acceptable.  dt_flash_fwd needs a workspace for the bf16 copies of
// K and V; this variant keeps that workspace in a fixed array that is part of
// the library's device image, so a call allocates nothing.  Q is read as fp32
// and rounded inside the attention kernel, exactly as dt_flash_fwd does, so
// the two entry points return bit-identical results.
//
// Limits and behaviour:
//  * The array is kNoAllocScratchBytes (24 MiB) on every GPU that loads the
//    library, held until the process exits.  It fits B*T*H*D <= 6,291,456
//    elements (for example B=1, T=3072, H=16, D=128); larger problems are
//    rejected with DT_ERR_INVALID_ARGUMENT before anything is launched.
//  * All calls on a device share the one array, and it keeps whatever the last
//    call wrote.  Nothing in it has to start at zero (each call overwrites the
//    part it reads), so it is never cleared.  Calls whose kernels can overlap
//    on the GPU (different streams, no ordering between them) race on it; order
//    them on one stream or with events.
//  * The first call on a device, with that device current, looks up the
//    array's device address (cudaGetSymbolAddress) and caches it for the rest
//    of the process.  Make that first call before any stream capture.  The
//    cache assumes the device's primary context is never reset: after
//    cudaDeviceReset the cached address is stale, so do not call this entry
//    point again in a process that reset the device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[24u << 20];
constexpr size_t kNoAllocScratchBytes = sizeof(g_noalloc_scratch);

namespace {
constexpr int kMaxDevices = 64;
void* g_noalloc_addr[kMaxDevices] = {};

int noalloc_scratch(int dev, void** out) {
    if (dev < 0 || dev >= kMaxDevices) return fail(DT_ERR_UNSUPPORTED, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_noalloc_addr[dev] == nullptr) {
        void* ptr = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || ptr == nullptr)
            return fail(DT_ERR_CUDA, "cudaGetSymbolAddress(no-alloc scratch) failed: %s", cudaGetErrorString(e));
        g_noalloc_addr[dev] = ptr;
    }
    *out = g_noalloc_addr[dev];
    return DT_OK;
}
}  // namespace

int dt_flash_fwd_noalloc(const float* q, const float* k, const float* v, float* o, float* softmax_m,
                         float* softmax_l, int B, int T, int H, int D, float scale, int causal, void* stream) {
    t_last_error.clear();
    DT_TRY(check_flash_shape(B, T, H, D));
    if ((long long)B * T * H == 0) return DT_OK;
    if (!q || !k || !v || !o) return fail(DT_ERR_INVALID_ARGUMENT, "null q/k/v/o");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
        return fail(DT_ERR_INVALID_ARGUMENT, "q/k/v/o must be 16-byte aligned");
    const long long n = (long long)B * T * H * D;
    const size_t one = align256((size_t)n * 2);
    if (2 * one > kNoAllocScratchBytes)
        return fail(DT_ERR_INVALID_ARGUMENT,
                    "dt_flash_fwd_noalloc: B*T*H*D = %lld exceeds the fixed scratch (at most %zu elements); "
                    "use dt_flash_fwd with a caller workspace",
                    n, kNoAllocScratchBytes / 4);
    int dev;
    DT_TRY(prepare_device(&dev));
    void* scratch;
    DT_TRY(noalloc_scratch(dev, &scratch));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    uint8_t* ws = reinterpret_cast<uint8_t*>(scratch);
    // K and V to bf16 in the fixed scratch; the attention kernel reads the fp32 Q rows itself
    DT_TRY(launch_cast3(k, v, nullptr, ws, ws + one, nullptr, n, st, 2));
    return launch_flash(nullptr, ws, ws + one, o, 0, (long long)H * D, softmax_m, softmax_l, nullptr, B, T, H, scale,
                        causal, st, Scatter(), q);
}

int dt_flash_fwd_bf16(const void* q, const void* k, const void* v, void* o, int o_bf16, long long o_row_stride,
                      float* softmax_m, float* softmax_l, const int* seq_lens, int B, int T, int H, int D,
                      float scale, int causal, void* stream) {
    t_last_error.clear();
    DT_TRY(check_flash_shape(B, T, H, D));
    if ((long long)B * T * H == 0) return DT_OK;
    if (!q || !k || !v || !o) return fail(DT_ERR_INVALID_ARGUMENT, "null q/k/v/o");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
        return fail(DT_ERR_INVALID_ARGUMENT, "q/k/v/o must be 16-byte aligned");
    if (o_row_stride < (long long)H * D || (o_row_stride % 8) != 0)
        return fail(DT_ERR_INVALID_ARGUMENT, "o_row_stride must be >= H*D and a multiple of 8");
    int dev;
    DT_TRY(prepare_device(&dev));
    return launch_flash(q, k, v, o, o_bf16 ? 1 : 0, o_row_stride, softmax_m, softmax_l, seq_lens, B, T, H, scale,
                        causal, reinterpret_cast<cudaStream_t>(stream));
}

int dt_flash_fwd_bf16_exchange(const void* q, const void* k, const void* v, void* const* recv_bufs, int ranks,
                               int rank, long long tokens_per_rank, float* softmax_m, float* softmax_l, int B, int T,
                               int H, int D, float scale, int causal, void* stream) {
    t_last_error.clear();
    DT_TRY(check_flash_shape(B, T, H, D));
    if ((long long)B * T * H == 0) return DT_OK;
    if (ranks < 1 || ranks > 8 || rank < 0 || rank >= ranks)
        return fail(DT_ERR_INVALID_ARGUMENT, "ranks must be 1..8 and 0 <= rank < ranks");
    if (!recv_bufs || tokens_per_rank <= 0 || tokens_per_rank * ranks != (long long)B * T)
        return fail(DT_ERR_INVALID_ARGUMENT, "tokens_per_rank * ranks must equal B*T");
    if (!q || !k || !v || !aligned16(q) || !aligned16(k) || !aligned16(v))
        return fail(DT_ERR_INVALID_ARGUMENT, "q/k/v must be non-null and 16-byte aligned");
    for (int r = 0; r < ranks; ++r)
        if (!recv_bufs[r] || !aligned16(recv_bufs[r]))
            return fail(DT_ERR_INVALID_ARGUMENT, "receive buffer %d must be non-null and 16-byte aligned", r);
    int dev;
    DT_TRY(prepare_device(&dev));
    Scatter sc;
    sc.ranks = ranks;
    sc.plane = rank;
    sc.tokens_per_rank = tokens_per_rank;
    sc.dst = recv_bufs;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    DT_TRY(launch_flash(q, k, v, nullptr, 1, (long long)H * D, softmax_m, softmax_l, nullptr, B, T, H, scale, causal,
                        st, sc));
    dt::elem::system_fence_kernel<<<1, 32, 0, st>>>();
    DT_CUDA(cudaGetLastError());
    return DT_OK;
}

int dt_flash_fwd_qf32(const float* q, const void* k, const void* v, void* o, int o_bf16, long long o_row_stride,
                      float* softmax_m, float* softmax_l, const int* seq_lens, int B, int T, int H, int D,
                      float scale, int causal, void* stream) {
    t_last_error.clear();
    DT_TRY(check_flash_shape(B, T, H, D));
    if ((long long)B * T * H == 0) return DT_OK;
    if (!q || !k || !v || !o) return fail(DT_ERR_INVALID_ARGUMENT, "null q/k/v/o");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
        return fail(DT_ERR_INVALID_ARGUMENT, "q/k/v/o must be 16-byte aligned");
    if (o_row_stride < (long long)H * D || (o_row_stride % 8) != 0)
        return fail(DT_ERR_INVALID_ARGUMENT, "o_row_stride must be >= H*D and a multiple of 8");
    int dev;
    DT_TRY(prepare_device(&dev));
    return launch_flash(nullptr, k, v, o, o_bf16 ? 1 : 0, o_row_stride, softmax_m, softmax_l, seq_lens, B, T, H,
                        scale, causal, reinterpret_cast<cudaStream_t>(stream), Scatter(), q);
}

int dt_flash_fwd_qf32_exchange(const float* q, const void* k, const void* v, void* const* recv_bufs, int ranks,
                               int rank, long long tokens_per_rank, float* softmax_m, float* softmax_l, int B, int T,
                               int H, int D, float scale, int causal, void* stream) {
    t_last_error.clear();
    DT_TRY(check_flash_shape(B, T, H, D));
    if ((long long)B * T * H == 0) return DT_OK;
    if (ranks < 1 || ranks > 8 || rank < 0 || rank >= ranks)
        return fail(DT_ERR_INVALID_ARGUMENT, "ranks must be 1..8 and 0 <= rank < ranks");
    if (!recv_bufs || tokens_per_rank <= 0 || tokens_per_rank * ranks != (long long)B * T)
        return fail(DT_ERR_INVALID_ARGUMENT, "tokens_per_rank * ranks must equal B*T");
    if (!q || !k || !v || !aligned16(q) || !aligned16(k) || !aligned16(v))
        return fail(DT_ERR_INVALID_ARGUMENT, "q/k/v must be non-null and 16-byte aligned");
    for (int r = 0; r < ranks; ++r)
        if (!recv_bufs[r] || !aligned16(recv_bufs[r]))
            return fail(DT_ERR_INVALID_ARGUMENT, "receive buffer %d must be non-null and 16-byte aligned", r);
    int dev;
    DT_TRY(prepare_device(&dev));
    Scatter sc;
    sc.ranks = ranks;
    sc.plane = rank;
    sc.tokens_per_rank = tokens_per_rank;
    sc.dst = recv_bufs;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    DT_TRY(launch_flash(nullptr, k, v, nullptr, 1, (long long)H * D, softmax_m, softmax_l, nullptr, B, T, H, scale,
                        causal, st, sc, q));
    dt::elem::system_fence_kernel<<<1, 32, 0, st>>>();
    DT_CUDA(cudaGetLastError());
    return DT_OK;
}

int dt_exchange_barrier(void* const* flag_bufs, int ranks, int rank, unsigned epoch, void* stream) {
    t_last_error.clear();
    if (ranks < 1 || ranks > 8 || rank < 0 || rank >= ranks)
        return fail(DT_ERR_INVALID_ARGUMENT, "ranks must be 1..8 and 0 <= rank < ranks");
    if (!flag_bufs || epoch == 0) return fail(DT_ERR_INVALID_ARGUMENT, "need flag buffers and an epoch > 0");
    dt::elem::BarrierArgs args{};
    for (int r = 0; r < ranks; ++r) {
        if (!flag_bufs[r] || ((uintptr_t)flag_bufs[r] & 3u))
            return fail(DT_ERR_INVALID_ARGUMENT, "flag buffer %d must be non-null and 4-byte aligned", r);
        args.flags[r] = static_cast<unsigned*>(flag_bufs[r]);
    }
    args.ranks = ranks;
    args.rank = rank;
    args.epoch = epoch;
    int dev;
    DT_TRY(prepare_device(&dev));
    dt::elem::exchange_barrier_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(args);
    DT_CUDA(cudaGetLastError());
    return DT_OK;
}

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

int dt_ipc_get_handle(const void* dev_ptr, void* handle_out, size_t* offset_out) {
    t_last_error.clear();
    if (!dev_ptr || !handle_out || !offset_out) return fail(DT_ERR_INVALID_ARGUMENT, "null argument");
    // The handle names the whole allocation; a caching allocator may hand out
    // an interior pointer, so report its offset from the allocation base.
    static AddressRangeFn range = nullptr;
    if (!range) {
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", reinterpret_cast<void**>(&range), cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !range)
            return fail(DT_ERR_CUDA, "cuMemGetAddressRange unavailable");
    }
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
        return fail(DT_ERR_INVALID_ARGUMENT, "pointer is not a device allocation");
    cudaIpcMemHandle_t h;
    DT_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    std::memcpy(handle_out, &h, sizeof(h));
    *offset_out = reinterpret_cast<uintptr_t>(dev_ptr) - static_cast<uintptr_t>(base);
    return DT_OK;
}

int dt_ipc_open(const void* handle, size_t offset, void** dev_ptr_out) {
    t_last_error.clear();
    if (!handle || !dev_ptr_out) return fail(DT_ERR_INVALID_ARGUMENT, "null argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    DT_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
    *dev_ptr_out = static_cast<uint8_t*>(base) + offset;
    return DT_OK;
}

int dt_ipc_close(void* dev_ptr, size_t offset) {
    t_last_error.clear();
    if (!dev_ptr) return DT_OK;
    DT_CUDA(cudaIpcCloseMemHandle(static_cast<uint8_t*>(dev_ptr) - offset));
    return DT_OK;
}

int dt_cast_f32_bf16(const float* src, void* dst, long long n, void* stream) {
    t_last_error.clear();
    if (n < 0 || (n % 4) != 0) return fail(DT_ERR_INVALID_ARGUMENT, "n must be a non-negative multiple of 4");
    if (n == 0) return DT_OK;
    if (!src || !dst || !aligned16(src) || ((uintptr_t)dst & 7u))
        return fail(DT_ERR_INVALID_ARGUMENT, "src must be 16-byte and dst 8-byte aligned");
    return launch_cast(src, dst, n, reinterpret_cast<cudaStream_t>(stream));
}

int dt_cast2_f32_bf16(const float* src0, const float* src1, void* dst0, void* dst1, long long n, void* stream) {
    t_last_error.clear();
    if (n < 0 || (n % 4) != 0) return fail(DT_ERR_INVALID_ARGUMENT, "n must be a non-negative multiple of 4");
    if (n == 0) return DT_OK;
    if (!src0 || !src1 || !dst0 || !dst1 || !aligned16(src0) || !aligned16(src1) || ((uintptr_t)dst0 & 7u) ||
        ((uintptr_t)dst1 & 7u))
        return fail(DT_ERR_INVALID_ARGUMENT, "sources must be 16-byte and destinations 8-byte aligned");
    return launch_cast3(src0, src1, nullptr, dst0, dst1, nullptr, n, reinterpret_cast<cudaStream_t>(stream), 2);
}

int dt_gemm_bf16_tn(const void* A, const void* B, void* C, int c_bf16, int M, int N, int K, long long ldc,
                    void* stream) {
    t_last_error.clear();
    if (M < 0 || N < 0 || K <= 0 || (K % 8) != 0)
        return fail(DT_ERR_INVALID_ARGUMENT, "need M,N >= 0 and K > 0 with K %% 8 == 0 (M=%d N=%d K=%d)", M, N, K);
    if (M == 0 || N == 0) return DT_OK;
    if (!A || !B || !C || !aligned16(A) || !aligned16(B) || !aligned16(C))
        return fail(DT_ERR_INVALID_ARGUMENT, "A, B, C must be non-null and 16-byte aligned");
    if (ldc < N || (ldc % (c_bf16 ? 8 : 4)) != 0)
        return fail(DT_ERR_INVALID_ARGUMENT, "ldc must be >= N and keep rows 16-byte aligned");
    int dev;
    DT_TRY(prepare_device(&dev));
    return launch_gemm(A, B, C, c_bf16 ? 1 : 0, M, N, K, ldc, reinterpret_cast<cudaStream_t>(stream));
}

int dt_gemm_bf16(const void* A, int a_mn, const void* B, int b_mn, void* C, int c_mode, int M, int N, int K,
                 long long ldc, void* stream) {
    t_last_error.clear();
    if (M < 0 || N < 0 || K <= 0) return fail(DT_ERR_INVALID_ARGUMENT, "need M, N >= 0 and K > 0");
    if (c_mode < 0 || c_mode > 2) return fail(DT_ERR_INVALID_ARGUMENT, "c_mode must be 0 (store fp32), 1 (store bf16) or 2 (add fp32)");
    if (M == 0 || N == 0) return DT_OK;
    if ((!a_mn || !b_mn) && (K % 8) != 0) return fail(DT_ERR_INVALID_ARGUMENT, "K-major operands need K %% 8 == 0");
    if ((a_mn && (M % 8) != 0) || (b_mn && (N % 8) != 0))
        return fail(DT_ERR_INVALID_ARGUMENT, "an MN-major operand needs its M (or N) %% 8 == 0");
    if (!A || !B || !C || !aligned16(A) || !aligned16(B) || !aligned16(C))
        return fail(DT_ERR_INVALID_ARGUMENT, "A, B, C must be non-null and 16-byte aligned");
    if (ldc < N || (ldc % (c_mode == 1 ? 8 : 4)) != 0)
        return fail(DT_ERR_INVALID_ARGUMENT, "ldc must be >= N and keep rows 16-byte aligned");
    int dev;
    DT_TRY(prepare_device(&dev));
    return launch_gemm(A, B, C, c_mode == 1 ? 1 : 0, M, N, K, ldc, reinterpret_cast<cudaStream_t>(stream), 1,
                       c_mode == 2 ? dt::gemm::kAccum : dt::gemm::kStore, nullptr, 0, 0, a_mn ? 1 : 0, b_mn ? 1 : 0);
}

int dt_gemm_bf16_tn_planar(const void* A, int a_planes, const void* B, void* C, int c_bf16, int M, int N, int K,
                           long long ldc, void* stream) {
    t_last_error.clear();
    if (a_planes <= 0 || K <= 0 || (K % a_planes) != 0 || ((K / a_planes) % 64) != 0)
        return fail(DT_ERR_INVALID_ARGUMENT, "K=%d must split into %d planes of a multiple of 64", K, a_planes);
    if (M < 0 || N < 0) return fail(DT_ERR_INVALID_ARGUMENT, "negative shape");
    if (M == 0 || N == 0) return DT_OK;
    if (!A || !B || !C || !aligned16(A) || !aligned16(B) || !aligned16(C))
        return fail(DT_ERR_INVALID_ARGUMENT, "A, B, C must be non-null and 16-byte aligned");
    if (ldc < N || (ldc % (c_bf16 ? 8 : 4)) != 0)
        return fail(DT_ERR_INVALID_ARGUMENT, "ldc must be >= N and keep rows 16-byte aligned");
    int dev;
    DT_TRY(prepare_device(&dev));
    return launch_gemm(A, B, C, c_bf16 ? 1 : 0, M, N, K, ldc, reinterpret_cast<cudaStream_t>(stream), a_planes);
}

int dt_qk_norm_rope(const float* q, const float* k, const float* v, long long ld_in, const float* q_gain,
                    const float* k_gain, void* q_out, void* k_out, void* v_out, int B, int T, float eps,
                    float rope_theta, void* stream) {
    t_last_error.clear();
    if (B < 0 || T < 0) return fail(DT_ERR_INVALID_ARGUMENT, "negative shape");
    if (T > kMaxSeqLen) return fail(DT_ERR_INVALID_ARGUMENT, "T=%d exceeds max_seq_len %d", T, kMaxSeqLen);
    if ((long long)B * T == 0) return DT_OK;
    if (ld_in < 2048 || (ld_in % 4) != 0) return fail(DT_ERR_INVALID_ARGUMENT, "ld_in must be >= 2048, multiple of 4");
    if (!q || !k || !v || !q_gain || !k_gain || !q_out || !k_out || !v_out || !aligned16(q) || !aligned16(k) ||
        !aligned16(v) || !aligned16(q_gain) || !aligned16(k_gain) || !aligned16(q_out) || !aligned16(k_out) ||
        !aligned16(v_out))
        return fail(DT_ERR_INVALID_ARGUMENT, "all pointers must be non-null and 16-byte aligned");
    int dev;
    DT_TRY(prepare_device(&dev));
    const float *st, *ct;
    DT_TRY(ensure_rope(dev, rope_theta, &st, &ct));
    return launch_prologue(q, k, v, ld_in, q_gain, k_gain, st, ct, q_out, k_out, v_out, B, T, eps,
                           reinterpret_cast<cudaStream_t>(stream));
}

int dt_rope_tables(float* sin_out, float* cos_out, int max_seq, int head_dim, float theta) {
    t_last_error.clear();
    if (!sin_out || !cos_out || max_seq < 0 || head_dim <= 0 || (head_dim % 2) != 0)
        return fail(DT_ERR_INVALID_ARGUMENT, "bad rope table arguments");
    std::vector<float> s, c;
    rope_tables_host(s, c, max_seq, head_dim, (double)theta);
    std::memcpy(sin_out, s.data(), s.size() * 4);
    std::memcpy(cos_out, c.data(), c.size() * 4);
    return DT_OK;
}

// ---- attention layer -------------------------------------------------------

// The fp32 weights stay on the device as the master copy the training step
// updates (the reference keeps fp32 param<2> members, param.h:5-15); the bf16
// copies the tensor cores read are derived from it.
static int attn_upload(dt_attn* a, const dt_attn_weights* w) {
    const int d = w->d_model;
    const size_t dd = (size_t)d * d;
    DT_CUDA(cudaMalloc(&a->master, 4 * dd * 4));
    DT_CUDA(cudaMalloc(&a->wqkv, 3 * dd * 2));
    DT_CUDA(cudaMalloc(&a->wo, dd * 2));
    DT_CUDA(cudaMalloc(&a->qg, (size_t)d * 4));
    DT_CUDA(cudaMalloc(&a->kg, (size_t)d * 4));
    const float* src[4] = {w->q_proj, w->k_proj, w->v_proj, w->o_proj};
    __nv_bfloat16* dst[4] = {a->wqkv, a->wqkv + dd, a->wqkv + 2 * dd, a->wo};
    for (int i = 0; i < 4; ++i) {
        DT_CUDA(cudaMemcpy(a->master + i * dd, src[i], dd * 4, cudaMemcpyHostToDevice));
        DT_TRY(launch_cast(a->master + i * dd, dst[i], (long long)dd, nullptr));
    }
    DT_CUDA(cudaDeviceSynchronize());
    DT_CUDA(cudaMemcpy(a->qg, w->q_norm, (size_t)d * 4, cudaMemcpyHostToDevice));
    DT_CUDA(cudaMemcpy(a->kg, w->k_norm, (size_t)d * 4, cudaMemcpyHostToDevice));
    return DT_OK;
}

int dt_attn_create(const dt_attn_weights* w, int device, dt_attn** out) {
    t_last_error.clear();
    if (!w || !out) return fail(DT_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    if (!w->q_proj || !w->k_proj || !w->v_proj || !w->o_proj || !w->q_norm || !w->k_norm)
        return fail(DT_ERR_INVALID_ARGUMENT, "null weight pointer");
    if (w->d_model != 2048 || w->n_heads <= 0 || w->d_model % w->n_heads != 0 || w->d_model / w->n_heads != 128)
        return fail(DT_ERR_UNSUPPORTED, "need d_model 2048 and head_dim 128 (got d_model=%d n_heads=%d)", w->d_model,
                    w->n_heads);
    DeviceGuard dg;
    DT_TRY(dg.enter(device));
    int dev;
    DT_TRY(prepare_device(&dev));
    dt_attn* a = new dt_attn();
    a->device = device;
    a->d_model = w->d_model;
    a->n_heads = w->n_heads;
    a->eps = w->eps;
    a->theta = w->rope_theta;
    int s = attn_upload(a, w);
    if (s == DT_OK) {
        const float *st, *ct;
        s = ensure_rope(dev, a->theta, &st, &ct);
    }
    if (s != DT_OK) {
        std::string msg = t_last_error;
        dt_attn_destroy(a);
        t_last_error = msg;
        return s;
    }
    *out = a;
    return DT_OK;
}

// Minimal .npy reader (format version 1.x/2.x/3.x, '<f4', C order), for the
// checkpoint files OlmoAttention.cpp:39-46 loads with xt::load_npy.
static int read_npy_f32(const std::string& path, std::vector<float>& data, std::vector<long long>& shape) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return fail(DT_ERR_IO, "cannot open %s", path.c_str());
    unsigned char magic[8];
    if (std::fread(magic, 1, 8, f) != 8 || std::memcmp(magic, "\x93NUMPY", 6) != 0) {
        std::fclose(f);
        return fail(DT_ERR_IO, "%s is not a .npy file", path.c_str());
    }
    size_t hlen = 0;
    if (magic[6] == 1) {
        unsigned char b[2];
        if (std::fread(b, 1, 2, f) != 2) { std::fclose(f); return fail(DT_ERR_IO, "%s: truncated", path.c_str()); }
        hlen = b[0] | (b[1] << 8);
    } else {
        unsigned char b[4];
        if (std::fread(b, 1, 4, f) != 4) { std::fclose(f); return fail(DT_ERR_IO, "%s: truncated", path.c_str()); }
        hlen = b[0] | (b[1] << 8) | (b[2] << 16) | ((size_t)b[3] << 24);
    }
    std::string header(hlen, '\0');
    if (std::fread(&header[0], 1, hlen, f) != hlen) {
        std::fclose(f);
        return fail(DT_ERR_IO, "%s: truncated header", path.c_str());
    }
    if (header.find("'descr': '<f4'") == std::string::npos || header.find("'fortran_order': False") == std::string::npos) {
        std::fclose(f);
        return fail(DT_ERR_IO, "%s: need little-endian float32 in C order", path.c_str());
    }
    shape.clear();
    const size_t lp = header.find('(', header.find("'shape'"));
    const size_t rp = header.find(')', lp);
    if (lp == std::string::npos || rp == std::string::npos) {
        std::fclose(f);
        return fail(DT_ERR_IO, "%s: no shape in header", path.c_str());
    }
    long long count = 1;
    for (size_t i = lp + 1; i < rp;) {
        while (i < rp && (header[i] == ' ' || header[i] == ',')) ++i;
        if (i >= rp) break;
        long long v = 0;
        while (i < rp && header[i] >= '0' && header[i] <= '9') v = v * 10 + (header[i++] - '0');
        shape.push_back(v);
        count *= v;
    }
    data.resize((size_t)count);
    const size_t got = std::fread(data.data(), 4, (size_t)count, f);
    std::fclose(f);
    if (got != (size_t)count) return fail(DT_ERR_IO, "%s: expected %lld floats, read %zu", path.c_str(), count, got);
    return DT_OK;
}

// The six weight files of attention layer `index` (OlmoAttention.cpp:39-46).
static int read_attn_npy(const char* folder, unsigned index, std::vector<float> (&buf)[6]) {
    const char* names[6] = {"q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm"};
    for (int i = 0; i < 6; ++i) {
        std::vector<long long> shape;
        const std::string path = std::string(folder) + "/model.layers." + std::to_string(index) + ".self_attn." +
                                 names[i] + ".weight.npy";
        DT_TRY(read_npy_f32(path, buf[i], shape));
        const bool ok = (i < 4) ? (shape.size() == 2 && shape[0] == 2048 && shape[1] == 2048)
                                : (shape.size() == 1 && shape[0] == 2048);
        if (!ok) return fail(DT_ERR_IO, "%s: unexpected shape", path.c_str());
    }
    return DT_OK;
}

int dt_attn_create_from_npy(const char* folder, unsigned index, int device, dt_attn** out) {
    t_last_error.clear();
    if (!folder || !out) return fail(DT_ERR_INVALID_ARGUMENT, "null argument");
    std::vector<float> buf[6];
    DT_TRY(read_attn_npy(folder, index, buf));
    dt_attn_weights w;
    w.q_proj = buf[0].data();
    w.k_proj = buf[1].data();
    w.v_proj = buf[2].data();
    w.o_proj = buf[3].data();
    w.q_norm = buf[4].data();
    w.k_norm = buf[5].data();
    w.d_model = 2048;
    w.n_heads = 16;
    w.eps = 1e-6f;
    w.rope_theta = 500000.f;
    return dt_attn_create(&w, device, out);
}

// ---- head-sharded attention layer (several GPUs) ---------------------------

int dt_comm_unique_id(void* id_out) {
    t_last_error.clear();
    if (!id_out) return fail(DT_ERR_INVALID_ARGUMENT, "null argument");
    NcclApi* n;
    DT_TRY(need_nccl(&n));
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    ncclUniqueId id;
    const ncclResult_t r = n->GetUniqueId(&id);
    if (r != ncclSuccess) return fail(DT_ERR_NCCL, "ncclGetUniqueId: %s", n->GetErrorString(r));
    std::memcpy(id_out, &id, sizeof(id));
    return DT_OK;
}

int dt_comm_create(const void* id, int world, int rank, int device, int timeout_ms, dt_comm** out) {
    t_last_error.clear();
    if (!id || !out) return fail(DT_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    if (world < 1 || world > 8 || rank < 0 || rank >= world)
        return fail(DT_ERR_INVALID_ARGUMENT, "need 1 <= world <= 8 and 0 <= rank < world (world=%d rank=%d)", world,
                    rank);
    if (timeout_ms <= 0) return fail(DT_ERR_INVALID_ARGUMENT, "timeout_ms must be positive");
    NcclApi* n;
    DT_TRY(need_nccl(&n));
    DeviceGuard dg;
    DT_TRY(dg.enter(device));
    int dev;
    DT_TRY(prepare_device(&dev));
    dt_comm* c = new dt_comm();
    c->world = world;
    c->rank = rank;
    c->device = device;
    c->timeout_ms = timeout_ms;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    const ncclResult_t r = n->CommInitRankConfig(&c->comm, world, uid, rank, &cfg);
    const int st = nccl_done(c, r, "ncclCommInitRankConfig");
    if (st != DT_OK) {
        const std::string msg = t_last_error;
        if (c->comm) n->CommAbort(c->comm);
        delete c;
        t_last_error = msg;
        return st;
    }
    *out = c;
    return DT_OK;
}

int dt_comm_abort(dt_comm* c) {
    t_last_error.clear();
    if (!c) return DT_OK;
    if (c->comm) {
        NcclApi* n;
        DT_TRY(need_nccl(&n));
        n->CommAbort(c->comm);
        c->comm = nullptr;
    }
    return DT_OK;
}

int dt_comm_destroy(dt_comm* c) {
    t_last_error.clear();
    if (!c) return DT_OK;
    int st = DT_OK;
    if (c->comm) {
        NcclApi* n;
        DT_TRY(need_nccl(&n));
        DeviceGuard dg;
        DT_TRY(dg.enter(c->device));
        st = nccl_done(c, n->CommDestroy(c->comm), "ncclCommDestroy");
        c->comm = nullptr;
    }
    delete c;
    return st;
}

int dt_qk_sumsq(const float* q, const float* k, long long ld, int width, long long M, float* ss, void* stream) {
    t_last_error.clear();
    if (M < 0 || width <= 0 || (width % 4) != 0 || ld < width || (ld % 4) != 0)
        return fail(DT_ERR_INVALID_ARGUMENT, "need M >= 0, width a positive multiple of 4, ld >= width, ld %% 4 == 0");
    if (M == 0) return DT_OK;
    if (!q || !k || !ss || !aligned16(q) || !aligned16(k) || ((uintptr_t)ss & 7u))
        return fail(DT_ERR_INVALID_ARGUMENT, "q, k 16-byte aligned and ss 8-byte aligned, non-null");
    int dev;
    DT_TRY(prepare_device(&dev));
    return launch_sumsq(q, k, ld, width, M, ss, reinterpret_cast<cudaStream_t>(stream));
}

int dt_qk_norm_rope_shard(const float* q, const float* k, const float* v, long long ld_in, const float* ss,
                          const float* q_gain, const float* k_gain, int heads, void* q_out, void* k_out, void* v_out,
                          int B, int T, float eps, float rope_theta, void* stream) {
    t_last_error.clear();
    if (B < 0 || T < 0) return fail(DT_ERR_INVALID_ARGUMENT, "negative shape");
    if (T > kMaxSeqLen) return fail(DT_ERR_INVALID_ARGUMENT, "T=%d exceeds max_seq_len %d", T, kMaxSeqLen);
    if (heads != 1 && heads != 2 && heads != 4 && heads != 8 && heads != 16)
        return fail(DT_ERR_INVALID_ARGUMENT, "heads must be 1, 2, 4, 8 or 16");
    if ((long long)B * T == 0) return DT_OK;
    if (ld_in < heads * 128 || (ld_in % 4) != 0)
        return fail(DT_ERR_INVALID_ARGUMENT, "ld_in must be >= heads*128 and a multiple of 4");
    const void* ptrs[] = {q, k, v, q_gain, k_gain, q_out, k_out, v_out};
    for (const void* ptr : ptrs)
        if (!ptr || !aligned16(ptr)) return fail(DT_ERR_INVALID_ARGUMENT, "pointers must be non-null and 16-byte aligned");
    if (!ss || ((uintptr_t)ss & 7u)) return fail(DT_ERR_INVALID_ARGUMENT, "ss must be non-null and 8-byte aligned");
    int dev;
    DT_TRY(prepare_device(&dev));
    const float *st, *ct;
    DT_TRY(ensure_rope(dev, rope_theta, &st, &ct));
    return launch_prologue_shard(q, k, v, ld_in, ss, q_gain, k_gain, heads, st, ct, q_out, k_out, v_out, B, T, eps,
                                 reinterpret_cast<cudaStream_t>(stream));
}

static void shard_release(dt_attn* a) {
    ShardState* sh = a->shard;
    if (!sh) return;
    for (int b = 0; b < 3; ++b)
        for (int r = 0; r < 8; ++r)
            if (sh->opened[b][r]) cudaIpcCloseMemHandle(sh->peers[b][r]);
    for (int b = 0; b < 3; ++b) cudaFree(sh->recv[b]);
    delete sh;
    a->shard = nullptr;
}

// Receive buffers of the in-kernel exchange for M tokens, and every rank's
// mapping of every rank's buffers (handles all-gathered over NCCL).  Collective.
static int shard_setup_exchange(dt_attn* a, long long M, cudaStream_t st) {
    ShardState* sh = a->shard;
    dt_comm* c = sh->comm;
    if (sh->recv_tokens == M) return DT_OK;
    NcclApi* n;
    DT_TRY(need_nccl(&n));
    DT_CUDA(cudaStreamSynchronize(st));
    for (int b = 0; b < 3; ++b)
        for (int r = 0; r < 8; ++r)
            if (sh->opened[b][r]) {
                DT_CUDA(cudaIpcCloseMemHandle(sh->peers[b][r]));
                sh->opened[b][r] = false;
            }
    for (int b = 0; b < 3; ++b) {
        DT_CUDA(cudaFree(sh->recv[b]));
        sh->recv[b] = nullptr;
    }
    sh->recv_tokens = 0;
    const size_t bytes = align256((size_t)M * sh->heads * 128 * 2);
    for (int b = 0; b < 2; ++b) DT_CUDA(cudaMalloc(&sh->recv[b], bytes));
    DT_CUDA(cudaMalloc(&sh->recv[2], 256));
    DT_CUDA(cudaMemset(sh->recv[2], 0, 256));
    const int G = c->world;
    // my three handles -> device -> all-gather -> host
    constexpr size_t kH = sizeof(cudaIpcMemHandle_t);
    std::vector<uint8_t> mine(3 * kH), all((size_t)G * 3 * kH);
    for (int b = 0; b < 3; ++b) {
        cudaIpcMemHandle_t h;
        DT_CUDA(cudaIpcGetMemHandle(&h, sh->recv[b]));
        std::memcpy(mine.data() + b * kH, &h, kH);
    }
    uint8_t* dbuf = nullptr;
    DT_CUDA(cudaMalloc(&dbuf, (size_t)(G + 1) * 3 * kH));
    int rc = DT_OK;
    if (cudaMemcpy(dbuf, mine.data(), 3 * kH, cudaMemcpyHostToDevice) != cudaSuccess) rc = DT_ERR_CUDA;
    if (rc == DT_OK)
        rc = nccl_done(c, n->AllGather(dbuf, dbuf + 3 * kH, 3 * kH, ncclUint8, c->comm, st), "ncclAllGather(handles)");
    if (rc == DT_OK && cudaStreamSynchronize(st) != cudaSuccess) rc = DT_ERR_CUDA;
    if (rc == DT_OK && cudaMemcpy(all.data(), dbuf + 3 * kH, all.size(), cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = DT_ERR_CUDA;
    cudaFree(dbuf);
    if (rc == DT_ERR_CUDA) return fail(DT_ERR_CUDA, "exchanging the receive-buffer handles failed");
    if (rc != DT_OK) return rc;
    for (int b = 0; b < 3; ++b)
        for (int r = 0; r < G; ++r) {
            if (r == c->rank) {
                sh->peers[b][r] = sh->recv[b];
                continue;
            }
            cudaIpcMemHandle_t h;
            std::memcpy(&h, all.data() + ((size_t)r * 3 + b) * kH, kH);
            DT_CUDA(cudaIpcOpenMemHandle(&sh->peers[b][r], h, cudaIpcMemLazyEnablePeerAccess));
            sh->opened[b][r] = true;
        }
    sh->recv_tokens = M;
    return DT_OK;
}

int dt_attn_create_sharded(const dt_attn_weights* w, dt_comm* comm, int exchange, dt_attn** out) {
    t_last_error.clear();
    if (!w || !out) return fail(DT_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    DT_TRY(comm_ok(comm));
    if (exchange != 0 && exchange != 1) return fail(DT_ERR_INVALID_ARGUMENT, "exchange must be 0 (in-kernel) or 1 (NCCL)");
    if (!w->q_proj || !w->k_proj || !w->v_proj || !w->o_proj || !w->q_norm || !w->k_norm)
        return fail(DT_ERR_INVALID_ARGUMENT, "null weight pointer");
    if (w->d_model != 2048 || w->n_heads != 16)
        return fail(DT_ERR_UNSUPPORTED, "need d_model 2048 and 16 heads of 128 (got d_model=%d n_heads=%d)",
                    w->d_model, w->n_heads);
    const int G = comm->world;
    if (16 % G != 0) return fail(DT_ERR_UNSUPPORTED, "16 heads do not split over %d ranks", G);
    DeviceGuard dg;
    DT_TRY(dg.enter(comm->device));
    int dev;
    DT_TRY(prepare_device(&dev));
    dt_attn* a = new dt_attn();
    a->device = comm->device;
    a->d_model = 2048;
    a->n_heads = 16;
    a->eps = w->eps;
    a->theta = w->rope_theta;
    a->shard = new ShardState();
    ShardState* sh = a->shard;
    sh->comm = comm;
    sh->exchange = exchange;
    sh->heads = 16 / G;
    sh->h0 = comm->rank * sh->heads;
    const size_t d = 2048, wcols = (size_t)sh->heads * 128, dd = d * d;
    auto cleanup = [&](int code) {
        const std::string msg = t_last_error;
        dt_attn_destroy(a);
        t_last_error = msg;
        return code;
    };
    // [Wq_r; Wk_r; Wv_r]: this rank's head rows of each projection, then all of Wo, staged
    // in fp32 one after the other in a buffer that holds the larger of the two
    float* stage = nullptr;
    const size_t stage_floats = std::max(3 * wcols * d, dd);
    if (cudaMalloc(&stage, stage_floats * 4) != cudaSuccess || cudaMalloc(&a->wqkv, 3 * wcols * d * 2) != cudaSuccess ||
        cudaMalloc(&a->wo, dd * 2) != cudaSuccess || cudaMalloc(&a->qg, d * 4) != cudaSuccess ||
        cudaMalloc(&a->kg, d * 4) != cudaSuccess) {
        cudaFree(stage);
        return cleanup(fail(DT_ERR_OUT_OF_MEMORY, "cudaMalloc failed for the sharded layer's weights"));
    }
    const float* src[3] = {w->q_proj, w->k_proj, w->v_proj};
    int rc = DT_OK;
    cudaError_t ce = cudaSuccess;
    for (int i = 0; i < 3 && ce == cudaSuccess; ++i)
        ce = cudaMemcpy(stage + i * wcols * d, src[i] + (size_t)sh->h0 * 128 * d, wcols * d * 4,
                        cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) rc = fail(DT_ERR_CUDA, "weight upload failed: %s", cudaGetErrorString(ce));
    if (rc == DT_OK) rc = launch_cast(stage, a->wqkv, (long long)(3 * wcols * d), nullptr);
    if (rc == DT_OK && (ce = cudaDeviceSynchronize()) != cudaSuccess)
        rc = fail(DT_ERR_CUDA, "weight cast failed: %s", cudaGetErrorString(ce));
    if (rc == DT_OK && (ce = cudaMemcpy(stage, w->o_proj, dd * 4, cudaMemcpyHostToDevice)) != cudaSuccess)
        rc = fail(DT_ERR_CUDA, "weight upload failed: %s", cudaGetErrorString(ce));
    if (rc == DT_OK) rc = launch_cast(stage, a->wo, (long long)dd, nullptr);
    if (rc == DT_OK && (ce = cudaDeviceSynchronize()) != cudaSuccess)
        rc = fail(DT_ERR_CUDA, "weight cast failed: %s", cudaGetErrorString(ce));
    cudaFree(stage);
    if (rc == DT_OK && ((ce = cudaMemcpy(a->qg, w->q_norm, d * 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
                        (ce = cudaMemcpy(a->kg, w->k_norm, d * 4, cudaMemcpyHostToDevice)) != cudaSuccess))
        rc = fail(DT_ERR_CUDA, "gain upload failed: %s", cudaGetErrorString(ce));
    if (rc == DT_OK) {
        const float *st, *ct;
        rc = ensure_rope(dev, a->theta, &st, &ct);
    }
    if (rc != DT_OK) return cleanup(rc);
    *out = a;
    return DT_OK;
}

// Workspace of a sharded forward for M tokens (w = this rank's columns):
// x bf16 [M, 2048] | [q|k|v] fp32 [M, 3w] | sums of squares [M, 2] fp32 |
// q, k, v bf16 [M, w] | exchange 1: local output and receive buffer bf16 [M, w] each
static size_t shard_ws_bytes(long long M, int w) {
    return align256(M * 2048 * 2) + align256(M * 3 * w * 4) + align256(M * 8) + 3 * align256(M * w * 2) +
           2 * align256(M * w * 2);
}

int dt_attn_forward_sharded(dt_attn* a, const float* x, int B, int T, const int* seq_lens, int gather, float* y,
                            void* stream) {
    t_last_error.clear();
    if (!a || !a->shard) return fail(DT_ERR_INVALID_ARGUMENT, "not a sharded handle (dt_attn_create_sharded)");
    ShardState* sh = a->shard;
    dt_comm* c = sh->comm;
    DT_TRY(comm_ok(c));
    if (B < 0 || T < 0) return fail(DT_ERR_INVALID_ARGUMENT, "negative shape");
    if (T > kMaxSeqLen) return fail(DT_ERR_INVALID_ARGUMENT, "T=%d exceeds max_seq_len %d", T, kMaxSeqLen);
    const long long M = (long long)B * T;
    const int G = c->world;
    if (M % G != 0) return fail(DT_ERR_INVALID_ARGUMENT, "B*T = %lld is not divisible by %d ranks", M, G);
    if (M == 0) return DT_OK;
    if (!x || !y || !aligned16(x) || !aligned16(y)) return fail(DT_ERR_INVALID_ARGUMENT, "x/y must be 16-byte aligned");
    NcclApi* n;
    DT_TRY(need_nccl(&n));
    DeviceGuard dg;
    DT_TRY(dg.enter(a->device));
    int dev;
    DT_TRY(prepare_device(&dev));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int w = sh->heads * 128;
    const long long tpr = M / G;
    const size_t need = shard_ws_bytes(M, w);
    if (a->ws_bytes < need) {
        DT_CUDA(cudaStreamSynchronize(st));
        if (a->ws) DT_CUDA(cudaFree(a->ws));
        a->ws = nullptr;
        a->ws_bytes = 0;
        DT_CUDA(cudaMalloc(&a->ws, need));
        a->ws_bytes = need;
    }
    if (sh->exchange == 0 && G > 1) DT_TRY(shard_setup_exchange(a, M, st));
    uint8_t* p = reinterpret_cast<uint8_t*>(a->ws);
    void* xb = p;
    p += align256(M * 2048 * 2);
    float* qkv = reinterpret_cast<float*>(p);
    p += align256(M * 3 * w * 4);
    float* ss = reinterpret_cast<float*>(p);
    p += align256(M * 8);
    void* qb = p;
    void* kb = p + align256(M * w * 2);
    void* vb = p + 2 * align256(M * w * 2);
    p += 3 * align256(M * w * 2);
    void* o_local = p;
    void* recv_nccl = p + align256(M * w * 2);
    const float *sin_t, *cos_t;
    DT_TRY(ensure_rope(dev, a->theta, &sin_t, &cos_t));
    DT_TRY(launch_cast(x, xb, M * 2048, st));
    // [q|k|v]_r = x [Wq_r; Wk_r; Wv_r]^T (padding-only tiles skipped, as in the one-GPU layer)
    DT_TRY(launch_gemm(xb, a->wqkv, qkv, 0, (int)M, 3 * w, 2048, 3 * w, st, 1, dt::gemm::kStore, seq_lens, T, 0));
    // QK-RMSNorm over all 2048 columns: this rank's partial sums, summed over the ranks
    DT_TRY(launch_sumsq(qkv, qkv + w, 3 * w, w, M, ss, st));
    DT_TRY(nccl_done(c, n->AllReduce(ss, ss, (size_t)(2 * M), ncclFloat32, ncclSum, c->comm, st),
                     "ncclAllReduce(sums of squares)"));
    DT_TRY(launch_prologue_shard(qkv, qkv + w, qkv + 2 * w, 3 * w, ss, a->qg + sh->h0 * 128, a->kg + sh->h0 * 128,
                                 sh->heads, sin_t, cos_t, qb, kb, vb, B, T, a->eps, st));
    const float scale = 1.0f / std::sqrt(128.0f);
    const void* a_op;
    if (G == 1) {
        DT_TRY(launch_flash(qb, kb, vb, o_local, 1, w, nullptr, nullptr, seq_lens, B, T, sh->heads, scale, 1, st));
        a_op = o_local;
    } else if (sh->exchange == 0) {
        // attention stores each row into its owner's buffer; the flag barrier (a system
        // fence, then every rank's step counter into every rank's flags over NVLink, and a
        // bounded wait for all of them) orders every rank's stores before the owners'
        // projections
        const int buf = sh->step & 1;
        sh->step++;
        Scatter sc;
        sc.ranks = G;
        sc.plane = c->rank;
        sc.tokens_per_rank = tpr;
        sc.dst = sh->peers[buf];
        DT_TRY(launch_flash(qb, kb, vb, nullptr, 1, w, nullptr, nullptr, seq_lens, B, T, sh->heads, scale, 1, st, sc));
        dt::elem::BarrierArgs ba{};
        for (int r = 0; r < G; ++r) ba.flags[r] = static_cast<unsigned*>(sh->peers[2][r]);
        ba.ranks = G;
        ba.rank = c->rank;
        ba.epoch = sh->step;
        dt::elem::exchange_barrier_kernel<<<1, 32, 0, st>>>(ba);
        DT_CUDA(cudaGetLastError());
        a_op = sh->recv[buf];
    } else {
        // local [M, w] token-major = [G, tpr, w]: slice g goes to rank g, plane g of mine comes from rank g
        DT_TRY(launch_flash(qb, kb, vb, o_local, 1, w, nullptr, nullptr, seq_lens, B, T, sh->heads, scale, 1, st));
        const size_t cnt = (size_t)tpr * w * 2;  // bytes per slice
        DT_TRY(nccl_done(c, n->GroupStart(), "ncclGroupStart"));
        int rc = DT_OK;
        for (int r = 0; r < G && rc == DT_OK; ++r) {
            rc = nccl_done(c, n->Send(static_cast<uint8_t*>(o_local) + r * cnt, cnt, ncclUint8, r, c->comm, st),
                           "ncclSend");
            if (rc == DT_OK)
                rc = nccl_done(c, n->Recv(static_cast<uint8_t*>(recv_nccl) + r * cnt, cnt, ncclUint8, r, c->comm, st),
                               "ncclRecv");
        }
        const int rc2 = nccl_done(c, n->GroupEnd(), "ncclGroupEnd");
        if (rc != DT_OK) return rc;
        DT_TRY(rc2);
        a_op = recv_nccl;
    }
    // y_r = A_r Wo^T over this rank's token slice; A_r is planar over the G source ranks
    float* y_mine = gather ? y + (size_t)c->rank * tpr * 2048 : y;
    DT_TRY(launch_gemm(a_op, a->wo, y_mine, 0, (int)tpr, 2048, 2048, 2048, st, G));
    if (gather && G > 1)
        DT_TRY(nccl_done(c, n->AllGather(y_mine, y, (size_t)tpr * 2048, ncclFloat32, c->comm, st),
                         "ncclAllGather(token slices)"));
    return DT_OK;
}

int dt_attn_forward_sharded_host(dt_attn* a, const float* x, int B, int T, const int* seq_lens, int gather,
                                 float* y) {
    t_last_error.clear();
    if (!a || !a->shard) return fail(DT_ERR_INVALID_ARGUMENT, "not a sharded handle (dt_attn_create_sharded)");
    if (B < 0 || T < 0) return fail(DT_ERR_INVALID_ARGUMENT, "negative shape");
    const long long M = (long long)B * T;
    const int G = a->shard->comm ? a->shard->comm->world : 1;
    if (M % G != 0) return fail(DT_ERR_INVALID_ARGUMENT, "B*T = %lld is not divisible by %d ranks", M, G);
    if (M == 0) return DT_OK;
    if (!x || !y) return fail(DT_ERR_INVALID_ARGUMENT, "null x/y");
    DeviceGuard dg;
    DT_TRY(dg.enter(a->device));
    if (!a->stream) DT_CUDA(cudaStreamCreateWithFlags(&a->stream, cudaStreamNonBlocking));
    const long long out_rows = gather ? M : M / G;
    const size_t xb = align256((size_t)M * 2048 * 4), yb = align256((size_t)out_rows * 2048 * 4);
    const size_t need = xb + yb + align256((size_t)B * 4);
    if (a->io_bytes < need) {
        if (a->io) DT_CUDA(cudaFree(a->io));
        a->io = nullptr;
        a->io_bytes = 0;
        DT_CUDA(cudaMalloc(&a->io, need));
        a->io_bytes = need;
    }
    uint8_t* io = reinterpret_cast<uint8_t*>(a->io);
    float* dx = reinterpret_cast<float*>(io);
    float* dy = reinterpret_cast<float*>(io + xb);
    int* dl = reinterpret_cast<int*>(io + xb + yb);
    DT_CUDA(cudaMemcpyAsync(dx, x, (size_t)M * 2048 * 4, cudaMemcpyHostToDevice, a->stream));
    if (seq_lens) DT_CUDA(cudaMemcpyAsync(dl, seq_lens, (size_t)B * 4, cudaMemcpyHostToDevice, a->stream));
    DT_TRY(dt_attn_forward_sharded(a, dx, B, T, seq_lens ? dl : nullptr, gather, dy, a->stream));
    DT_CUDA(cudaMemcpyAsync(y, dy, (size_t)out_rows * 2048 * 4, cudaMemcpyDeviceToHost, a->stream));
    DT_CUDA(cudaStreamSynchronize(a->stream));
    bool had;
    return read_device_error(&had);
}

int dt_attn_create_sharded_from_npy(const char* folder, unsigned index, dt_comm* comm, int exchange, dt_attn** out) {
    t_last_error.clear();
    if (!folder || !out) return fail(DT_ERR_INVALID_ARGUMENT, "null argument");
    std::vector<float> buf[6];
    DT_TRY(read_attn_npy(folder, index, buf));
    dt_attn_weights w;
    w.q_proj = buf[0].data();
    w.k_proj = buf[1].data();
    w.v_proj = buf[2].data();
    w.o_proj = buf[3].data();
    w.q_norm = buf[4].data();
    w.k_norm = buf[5].data();
    w.d_model = 2048;
    w.n_heads = 16;
    w.eps = 1e-6f;
    w.rope_theta = 500000.f;
    return dt_attn_create_sharded(&w, comm, exchange, out);
}

int dt_attn_destroy(dt_attn* a) {
    if (!a) return DT_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(a->device);
    shard_release(a);
    cudaFree(a->wqkv);
    cudaFree(a->wo);
    cudaFree(a->qg);
    cudaFree(a->kg);
    cudaFree(a->ws);
    cudaFree(a->io);
    cudaFree(a->master);
    cudaFree(a->grad);
    cudaFree(a->bws);
    if (a->stream) cudaStreamDestroy(a->stream);
    cudaSetDevice(prev);
    delete a;
    return DT_OK;
}

// Scratch of attn_core for M tokens: [q|k|v] fp32 and four bf16 [M, d] arrays.
// [q|k|v] fp32, q/k/v/attention-output bf16, then softmax m and l ([M, 16] fp32 each)
static size_t attn_core_bytes(long long M) {
    return align256(M * 6144 * 4) + 4 * align256(M * 2048 * 2) + 2 * align256(M * 16 * 4);
}

// OlmoAttention::forward on a bf16 input (OlmoAttention.cpp:56-108): fused QKV
// GEMM, QK-norm + RoPE prologue, flash attention, O projection into y (fp32).
static int attn_core(dt_attn* a, const void* xb, int B, int T, const int* seq_lens, float* y, uint8_t* ws, int dev,
                     cudaStream_t st) {
    // With seq_lens, projection tiles made only of padding rows are skipped: the
    // QKV rows there are never read (attention stops at each sequence's length)
    // and the O projection writes zeros for them.
    const long long M = (long long)B * T;
    const int d = a->d_model;
    const size_t act = align256(M * d * 2);
    float* qkv = reinterpret_cast<float*>(ws);
    uint8_t* rest = ws + align256(M * 3 * d * 4);
    void* qb = rest;
    void* kb = rest + act;
    void* vb = rest + 2 * act;
    void* ab = rest + 3 * act;
    // the softmax statistics stay in the workspace for the backward
    float* sm_m = reinterpret_cast<float*>(rest + 4 * act);
    float* sm_l = reinterpret_cast<float*>(rest + 4 * act + align256(M * a->n_heads * 4));
    const float *sin_t, *cos_t;
    DT_TRY(ensure_rope(dev, a->theta, &sin_t, &cos_t));
    // [q|k|v] = x Wqkv^T: q and k in fp32 (the norm's input, kept for the backward), v
    // straight in bf16 (attention's operand; the prologue leaves it alone)
    DT_TRY(launch_gemm(xb, a->wqkv, qkv, 0, (int)M, 3 * d, d, 3 * d, st, 1, dt::gemm::kStore, seq_lens, T, 0, 0, 0,
                       vb, d, 2 * d));
    DT_TRY(launch_prologue(qkv, qkv + d, nullptr, 3 * d, a->qg, a->kg, sin_t, cos_t, qb, kb, vb, B, T, a->eps,
                           st));                                                    // norm + RoPE
    DT_TRY(launch_flash(qb, kb, vb, ab, 1, d, sm_m, sm_l, seq_lens, B, T, a->n_heads, 1.0f / std::sqrt(128.0f), 1,
                        st));                                                       // attention
    DT_TRY(launch_gemm(ab, a->wo, y, 0, (int)M, d, d, d, st, 1, dt::gemm::kStore, seq_lens, T,
                       1));                                                         // y = a Wo^T
    return DT_OK;
}

static int attn_workspace(dt_attn* a, long long M, uint8_t** ws) {
    const size_t need = align256(M * 2048 * 2) + attn_core_bytes(M);
    if (a->ws_bytes < need) {
        if (a->ws) DT_CUDA(cudaFree(a->ws));
        a->ws = nullptr;
        a->ws_bytes = 0;
        DT_CUDA(cudaMalloc(&a->ws, need));
        a->ws_bytes = need;
    }
    *ws = reinterpret_cast<uint8_t*>(a->ws);
    return DT_OK;
}

int dt_attn_forward(dt_attn* a, const float* x, int B, int T, const int* seq_lens, float* y, void* stream) {
    t_last_error.clear();
    if (!a) return fail(DT_ERR_INVALID_ARGUMENT, "null handle");
    if (a->shard) return fail(DT_ERR_UNSUPPORTED, "head-sharded handle: use dt_attn_forward_sharded");
    if (B < 0 || T < 0) return fail(DT_ERR_INVALID_ARGUMENT, "negative shape");
    if (T > kMaxSeqLen) return fail(DT_ERR_INVALID_ARGUMENT, "T=%d exceeds max_seq_len %d", T, kMaxSeqLen);
    const long long M = (long long)B * T;
    if (M == 0) return DT_OK;
    if (!x || !y || !aligned16(x) || !aligned16(y)) return fail(DT_ERR_INVALID_ARGUMENT, "x/y must be 16-byte aligned");
    DeviceGuard dg;
    DT_TRY(dg.enter(a->device));
    int dev;
    DT_TRY(prepare_device(&dev));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int d = a->d_model;
    uint8_t* ws;
    DT_TRY(attn_workspace(a, M, &ws));
    void* xb = ws;
    DT_TRY(launch_cast(x, xb, M * d, st));  // x -> bf16
    a->last_B = B;
    a->last_T = T;
    a->last_varlen = seq_lens != nullptr;
    return attn_core(a, xb, B, T, seq_lens, y, ws + align256(M * d * 2), dev, st);
}

int dt_attn_forward_host(dt_attn* a, const float* x, int B, int T, const int* seq_lens, float* y) {
    t_last_error.clear();
    if (!a) return fail(DT_ERR_INVALID_ARGUMENT, "null handle");
    if (a->shard) return fail(DT_ERR_UNSUPPORTED, "head-sharded handle: use dt_attn_forward_sharded");
    if (B < 0 || T < 0) return fail(DT_ERR_INVALID_ARGUMENT, "negative shape");
    const long long M = (long long)B * T;
    if (M == 0) return DT_OK;
    if (!x || !y) return fail(DT_ERR_INVALID_ARGUMENT, "null x/y");
    DeviceGuard dg;
    DT_TRY(dg.enter(a->device));
    if (!a->stream) DT_CUDA(cudaStreamCreateWithFlags(&a->stream, cudaStreamNonBlocking));
    const size_t xb = align256((size_t)M * a->d_model * 4);
    const size_t need = 2 * xb + align256((size_t)B * 4);
    if (a->io_bytes < need) {
        if (a->io) DT_CUDA(cudaFree(a->io));
        a->io = nullptr;
        a->io_bytes = 0;
        DT_CUDA(cudaMalloc(&a->io, need));
        a->io_bytes = need;
    }
    uint8_t* io = reinterpret_cast<uint8_t*>(a->io);
    float* dx = reinterpret_cast<float*>(io);
    float* dy = reinterpret_cast<float*>(io + xb);
    int* dl = reinterpret_cast<int*>(io + 2 * xb);
    DT_CUDA(cudaMemcpyAsync(dx, x, (size_t)M * a->d_model * 4, cudaMemcpyHostToDevice, a->stream));
    if (seq_lens) DT_CUDA(cudaMemcpyAsync(dl, seq_lens, (size_t)B * 4, cudaMemcpyHostToDevice, a->stream));
    DT_TRY(dt_attn_forward(a, dx, B, T, seq_lens ? dl : nullptr, dy, a->stream));
    DT_CUDA(cudaMemcpyAsync(y, dy, (size_t)M * a->d_model * 4, cudaMemcpyDeviceToHost, a->stream));
    DT_CUDA(cudaStreamSynchronize(a->stream));
    bool had;
    return read_device_error(&had);
}

// ---- training path: OlmoAttention::backward / step / zero_grad --------------
//
// The forward leaves in the handle's workspace exactly the activations the
// reference saves as members (OlmoAttention.h:28-38): bf16 x, the fp32 [q|k|v]
// projections before the norm, the bf16 q/k/v after norm and RoPE, the bf16
// attention output and the softmax statistics.  The backward of the last
// forward (same B, T; no seq_lens) runs as
//   dWo += dY^T A,  dA = dY Wo                       (OlmoAttention.cpp:194-209)
//   dQ, dK, dV = flash backward(dA, A, m, l, q, k, v) (:211-225)
//   RoPE^T and QK-RMSNorm backward -> [dq|dk|dv] bf16 (:227-237)
//   d[Wq;Wk;Wv] += [dq|dk|dv]^T x,  dX = [dq|dk|dv] [Wq;Wk;Wv]  (:239-298)
// with the gradients accumulated (beta = 1, as the reference) until zero_grad.

static int attn_grads(dt_attn* a) {
    if (a->grad) return DT_OK;
    const size_t d = (size_t)a->d_model;
    DT_CUDA(cudaMalloc(&a->grad, (4 * d * d + 2 * d) * 4));
    DT_CUDA(cudaMemset(a->grad, 0, (4 * d * d + 2 * d) * 4));
    return DT_OK;
}

int dt_attn_backward(dt_attn* a, const float* dy, int B, int T, float* dx, void* stream) {
    t_last_error.clear();
    if (!a) return fail(DT_ERR_INVALID_ARGUMENT, "null handle");
    if (a->shard) return fail(DT_ERR_UNSUPPORTED, "head-sharded handle: use dt_attn_forward_sharded");
    if (B != a->last_B || T != a->last_T || (long long)B * T == 0)
        return fail(DT_ERR_INVALID_ARGUMENT, "backward needs the shape of the last forward (B=%d T=%d), got B=%d T=%d",
                    a->last_B, a->last_T, B, T);
    if (a->last_varlen)
        return fail(DT_ERR_UNSUPPORTED, "backward of a forward with seq_lens (the reference has no padding mask)");
    if (!dy || !dx || !aligned16(dy) || !aligned16(dx))
        return fail(DT_ERR_INVALID_ARGUMENT, "dy/dx must be non-null and 16-byte aligned");
    DeviceGuard dg;
    DT_TRY(dg.enter(a->device));
    int dev;
    DT_TRY(prepare_device(&dev));
    DT_TRY(attn_grads(a));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const long long M = (long long)B * T;
    const int d = a->d_model, H = a->n_heads;
    const size_t dd = (size_t)d * d;
    // forward activations in the workspace (layout of dt_attn_forward / attn_core)
    uint8_t* ws = reinterpret_cast<uint8_t*>(a->ws);
    const void* xb = ws;
    uint8_t* core = ws + align256(M * d * 2);
    const float* qkv = reinterpret_cast<const float*>(core);
    uint8_t* rest = core + align256(M * 3 * d * 4);
    const size_t act = align256(M * d * 2);
    const void *qb = rest, *kb = rest + act, *vb = rest + 2 * act, *ab = rest + 3 * act;
    const float* sm_m = reinterpret_cast<const float*>(rest + 4 * act);
    const float* sm_l = reinterpret_cast<const float*>(rest + 4 * act + align256(M * H * 4));
    // scratch
    const size_t f32 = align256(M * d * 4), rows = flash_bwd_rows_bytes(B, T, H);
    const long long nparts = (M + dt::elem::kBwdRows - 1) / dt::elem::kBwdRows;
    const size_t need = act + f32 + act + 2 * rows + 3 * f32 + align256(M * 3 * d * 2) + align256(nparts * 2 * d * 4);
    if (a->bws_bytes < need) {
        if (a->bws) DT_CUDA(cudaFree(a->bws));
        a->bws = nullptr;
        a->bws_bytes = 0;
        DT_CUDA(cudaMalloc(&a->bws, need));
        a->bws_bytes = need;
    }
    uint8_t* w = reinterpret_cast<uint8_t*>(a->bws);
    void* dyb = w;
    float* da = reinterpret_cast<float*>(w + act);
    void* dob = w + act + f32;
    float* dvec = reinterpret_cast<float*>(w + 2 * act + f32);
    float* lse2 = reinterpret_cast<float*>(w + 2 * act + f32 + rows);
    float* dq = reinterpret_cast<float*>(w + 2 * act + f32 + 2 * rows);
    float* dk = dq + f32 / 4;
    float* dv = dk + f32 / 4;
    void* dqkv = w + 2 * act + 4 * f32 + 2 * rows;
    float* gain_part = reinterpret_cast<float*>(w + 2 * act + 4 * f32 + 2 * rows + align256(M * 3 * d * 2));
    float* g_qkv = a->grad;
    float* g_o = a->grad + 3 * dd;
    float* g_qn = a->grad + 4 * dd;
    float* g_kn = g_qn + d;
    DT_TRY(launch_cast(dy, dyb, M * d, st));
    DT_TRY(launch_gemm(dyb, ab, g_o, 0, d, d, (int)M, d, st, 1, dt::gemm::kAccum, nullptr, 0, 0, 1, 1));  // dWo += dY^T A
    DT_TRY(launch_gemm(dyb, a->wo, da, 0, (int)M, d, d, d, st, 1, dt::gemm::kStore, nullptr, 0, 0, 0, 1));  // dA = dY Wo
    DT_TRY(launch_flash_bwd(qb, kb, vb, da, nullptr, ab, d, sm_m, sm_l, dq, dk, dv, B, T, H, 1.0f / std::sqrt(128.0f), 1,
                            dob, dvec, lse2, st));
    const float *sin_t, *cos_t;
    DT_TRY(ensure_rope(dev, a->theta, &sin_t, &cos_t));
    dt::elem::NormRopeBwdParams np{};
    np.dq = dq;
    np.dk = dk;
    np.dv = dv;
    np.xq = qkv;
    np.xk = qkv + d;
    np.ld_x = 3 * d;
    np.q_gain = a->qg;
    np.k_gain = a->kg;
    np.sin_t = sin_t;
    np.cos_t = cos_t;
    np.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv);
    np.gain_part = gain_part;
    np.M = M;
    np.T = T;
    np.eps = a->eps;
    dt::elem::qk_norm_rope_bwd_kernel<<<(unsigned)nparts, dt::elem::kPrologueThreads, 0, st>>>(np);
    DT_CUDA(cudaGetLastError());
    dt::elem::gain_grad_reduce_kernel<<<(2 * d + 255) / 256, 256, 0, st>>>(gain_part, (int)nparts, g_qn, g_kn);
    DT_CUDA(cudaGetLastError());
    DT_TRY(launch_gemm(dqkv, xb, g_qkv, 0, 3 * d, d, (int)M, d, st, 1, dt::gemm::kAccum, nullptr, 0, 0, 1,
                       1));  // d[Wq;Wk;Wv] += [dq|dk|dv]^T x
    DT_TRY(launch_gemm(dqkv, a->wqkv, dx, 0, (int)M, d, 3 * d, d, st, 1, dt::gemm::kStore, nullptr, 0, 0, 0,
                       1));  // dX = [dq|dk|dv] [Wq;Wk;Wv]
    return DT_OK;
}

int dt_attn_backward_host(dt_attn* a, const float* dy, int B, int T, float* dx) {
    t_last_error.clear();
    if (!a) return fail(DT_ERR_INVALID_ARGUMENT, "null handle");
    if (a->shard) return fail(DT_ERR_UNSUPPORTED, "head-sharded handle: use dt_attn_forward_sharded");
    if (!dy || !dx) return fail(DT_ERR_INVALID_ARGUMENT, "null dy/dx");
    const long long M = (long long)B * T;
    if (M <= 0 || B != a->last_B || T != a->last_T)
        return fail(DT_ERR_INVALID_ARGUMENT, "backward needs the shape of the last forward (B=%d T=%d)", a->last_B,
                    a->last_T);
    DeviceGuard dg;
    DT_TRY(dg.enter(a->device));
    if (!a->stream) DT_CUDA(cudaStreamCreateWithFlags(&a->stream, cudaStreamNonBlocking));
    const size_t xb = align256((size_t)M * a->d_model * 4);
    if (a->io_bytes < 2 * xb) {
        if (a->io) DT_CUDA(cudaFree(a->io));
        a->io = nullptr;
        a->io_bytes = 0;
        DT_CUDA(cudaMalloc(&a->io, 2 * xb));
        a->io_bytes = 2 * xb;
    }
    uint8_t* io = reinterpret_cast<uint8_t*>(a->io);
    float* ddy = reinterpret_cast<float*>(io);
    float* ddx = reinterpret_cast<float*>(io + xb);
    DT_CUDA(cudaMemcpyAsync(ddy, dy, (size_t)M * a->d_model * 4, cudaMemcpyHostToDevice, a->stream));
    DT_TRY(dt_attn_backward(a, ddy, B, T, ddx, a->stream));
    DT_CUDA(cudaMemcpyAsync(dx, ddx, (size_t)M * a->d_model * 4, cudaMemcpyDeviceToHost, a->stream));
    DT_CUDA(cudaStreamSynchronize(a->stream));
    bool had;
    return read_device_error(&had);
}

int dt_attn_step(dt_attn* a, float lr, void* stream) {
    t_last_error.clear();
    if (!a) return fail(DT_ERR_INVALID_ARGUMENT, "null handle");
    if (a->shard) return fail(DT_ERR_UNSUPPORTED, "head-sharded handle: use dt_attn_forward_sharded");
    DeviceGuard dg;
    DT_TRY(dg.enter(a->device));
    DT_TRY(attn_grads(a));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const long long dd = (long long)a->d_model * a->d_model;
    dt::elem::sgd_kernel<<<148 * 8, 256, 0, st>>>(a->master, a->grad, a->wqkv, lr, 3 * dd);
    dt::elem::sgd_kernel<<<148 * 8, 256, 0, st>>>(a->master + 3 * dd, a->grad + 3 * dd, a->wo, lr, dd);
    dt::elem::sgd_kernel<<<8, 256, 0, st>>>(a->qg, a->grad + 4 * dd, nullptr, lr, a->d_model);
    dt::elem::sgd_kernel<<<8, 256, 0, st>>>(a->kg, a->grad + 4 * dd + a->d_model, nullptr, lr, a->d_model);
    DT_CUDA(cudaGetLastError());
    return DT_OK;
}

int dt_attn_zero_grad(dt_attn* a, void* stream) {
    t_last_error.clear();
    if (!a) return fail(DT_ERR_INVALID_ARGUMENT, "null handle");
    if (a->shard) return fail(DT_ERR_UNSUPPORTED, "head-sharded handle: use dt_attn_forward_sharded");
    DeviceGuard dg;
    DT_TRY(dg.enter(a->device));
    if (!a->grad) return DT_OK;
    const size_t d = (size_t)a->d_model;
    DT_CUDA(cudaMemsetAsync(a->grad, 0, (4 * d * d + 2 * d) * 4, reinterpret_cast<cudaStream_t>(stream)));
    return DT_OK;
}

int dt_attn_get_params_host(dt_attn* a, float* q_proj, float* k_proj, float* v_proj, float* o_proj, float* q_norm,
                            float* k_norm, int gradients) {
    t_last_error.clear();
    if (!a) return fail(DT_ERR_INVALID_ARGUMENT, "null handle");
    if (a->shard) return fail(DT_ERR_UNSUPPORTED, "head-sharded handle: use dt_attn_forward_sharded");
    DeviceGuard dg;
    DT_TRY(dg.enter(a->device));
    DT_CUDA(cudaDeviceSynchronize());
    const size_t d = (size_t)a->d_model, dd = d * d;
    if (gradients) DT_TRY(attn_grads(a));
    const float* base = gradients ? a->grad : a->master;
    float* outs[4] = {q_proj, k_proj, v_proj, o_proj};
    for (int i = 0; i < 4; ++i)
        if (outs[i]) DT_CUDA(cudaMemcpy(outs[i], base + i * dd, dd * 4, cudaMemcpyDeviceToHost));
    const float* qn = gradients ? a->grad + 4 * dd : a->qg;
    const float* kn = gradients ? a->grad + 4 * dd + d : a->kg;
    if (q_norm) DT_CUDA(cudaMemcpy(q_norm, qn, d * 4, cudaMemcpyDeviceToHost));
    if (k_norm) DT_CUDA(cudaMemcpy(k_norm, kn, d * 4, cudaMemcpyDeviceToHost));
    bool had;
    return read_device_error(&had);
}

// ---- full model prefill (configuration 3) ------------------------------------

struct dt_model {
    int device = 0;
    int n_layers = 0, vocab = 0, d_model = 0, n_heads = 0, hidden = 0;
    float eps = 1e-6f, theta = 500000.f;
    float* embed = nullptr;              // [vocab, d] fp32 (gathered into the fp32 residual stream)
    __nv_bfloat16* lm_head = nullptr;    // [vocab, d]
    float* final_norm = nullptr;         // [d]
    std::vector<dt_attn*> attn;          // per layer: Wqkv, Wo, q/k norm gains
    std::vector<float*> pa_norm, pf_norm;
    std::vector<__nv_bfloat16*> w_gu;    // [2*hidden, d], gate/up interleaved in 128-row blocks
    std::vector<__nv_bfloat16*> w_down;  // [d, hidden]
    void* ws = nullptr;
    size_t ws_bytes = 0;
    void* io = nullptr;
    size_t io_bytes = 0;
    cudaStream_t stream = nullptr;
};

static int upload_bf16(const float* host, size_t n, __nv_bfloat16** out, float* stage) {
    DT_CUDA(cudaMalloc(out, n * 2));
    DT_CUDA(cudaMemcpy(stage, host, n * 4, cudaMemcpyHostToDevice));
    DT_TRY(launch_cast(stage, *out, (long long)n, nullptr));
    DT_CUDA(cudaDeviceSynchronize());
    return DT_OK;
}

static int upload_f32(const float* host, size_t n, float** out) {
    DT_CUDA(cudaMalloc(out, n * 4));
    DT_CUDA(cudaMemcpy(*out, host, n * 4, cudaMemcpyHostToDevice));
    return DT_OK;
}

static int model_upload(dt_model* m, const dt_model_weights* w) {
    const int d = m->d_model, hid = m->hidden;
    const size_t stage_n = std::max((size_t)m->vocab * d, (size_t)2 * hid * d);
    float* stage = nullptr;
    DT_CUDA(cudaMalloc(&stage, stage_n * 4));
    int s = DT_OK;
    do {
        if ((s = upload_f32(w->embed, (size_t)m->vocab * d, &m->embed)) != DT_OK) break;
        if ((s = upload_bf16(w->lm_head, (size_t)m->vocab * d, &m->lm_head, stage)) != DT_OK) break;
        if ((s = upload_f32(w->final_norm, d, &m->final_norm)) != DT_OK) break;
        for (int l = 0; l < m->n_layers && s == DT_OK; ++l) {
            const dt_model_layer_weights& L = w->layers[l];
            dt_attn_weights aw;
            aw.q_proj = L.q_proj;
            aw.k_proj = L.k_proj;
            aw.v_proj = L.v_proj;
            aw.o_proj = L.o_proj;
            aw.q_norm = L.q_norm;
            aw.k_norm = L.k_norm;
            aw.d_model = d;
            aw.n_heads = m->n_heads;
            aw.eps = m->eps;
            aw.rope_theta = m->theta;
            dt_attn* a = nullptr;
            if ((s = dt_attn_create(&aw, m->device, &a)) != DT_OK) break;
            m->attn.push_back(a);
            float *pa = nullptr, *pf = nullptr;
            if ((s = upload_f32(L.post_attention_norm, d, &pa)) != DT_OK) break;
            m->pa_norm.push_back(pa);
            if ((s = upload_f32(L.post_feedforward_norm, d, &pf)) != DT_OK) break;
            m->pf_norm.push_back(pf);
            // gate/up interleaved by 128-row blocks: rows [256b, 256b+128) = gate block b,
            // rows [256b+128, 256b+256) = up block b
            const size_t blk = (size_t)128 * d;
            cudaError_t e = cudaMemcpy2D(stage, 2 * blk * 4, L.gate_proj, blk * 4, blk * 4, hid / 128,
                                         cudaMemcpyHostToDevice);
            if (e == cudaSuccess)
                e = cudaMemcpy2D(stage + blk, 2 * blk * 4, L.up_proj, blk * 4, blk * 4, hid / 128,
                                 cudaMemcpyHostToDevice);
            if (e != cudaSuccess) { s = fail(DT_ERR_CUDA, "uploading MLP weights: %s", cudaGetErrorString(e)); break; }
            __nv_bfloat16* gu = nullptr;
            e = cudaMalloc(&gu, (size_t)2 * hid * d * 2);
            if (e != cudaSuccess) { s = fail(DT_ERR_OUT_OF_MEMORY, "cudaMalloc: %s", cudaGetErrorString(e)); break; }
            m->w_gu.push_back(gu);
            if ((s = launch_cast(stage, gu, (long long)2 * hid * d, nullptr)) != DT_OK) break;
            __nv_bfloat16* dn = nullptr;
            if ((s = upload_bf16(L.down_proj, (size_t)d * hid, &dn, stage)) != DT_OK) break;
            m->w_down.push_back(dn);
        }
    } while (false);
    cudaDeviceSynchronize();
    cudaFree(stage);
    return s;
}

int dt_model_destroy(dt_model* m) {
    if (!m) return DT_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(m->device);
    for (dt_attn* a : m->attn) dt_attn_destroy(a);
    for (float* x : m->pa_norm) cudaFree(x);
    for (float* x : m->pf_norm) cudaFree(x);
    for (__nv_bfloat16* x : m->w_gu) cudaFree(x);
    for (__nv_bfloat16* x : m->w_down) cudaFree(x);
    cudaFree(m->embed);
    cudaFree(m->lm_head);
    cudaFree(m->final_norm);
    cudaFree(m->ws);
    cudaFree(m->io);
    if (m->stream) cudaStreamDestroy(m->stream);
    cudaSetDevice(prev);
    delete m;
    return DT_OK;
}

int dt_model_create(const dt_model_weights* w, int device, dt_model** out) {
    t_last_error.clear();
    if (!w || !out) return fail(DT_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    if (w->d_model != 2048 || w->n_heads <= 0 || w->d_model / w->n_heads != 128 || w->d_model % w->n_heads)
        return fail(DT_ERR_UNSUPPORTED, "need d_model 2048 and head_dim 128");
    if (w->n_layers <= 0 || w->vocab <= 0 || w->hidden <= 0 || (w->hidden % 128) != 0 || (w->vocab % 8) != 0)
        return fail(DT_ERR_INVALID_ARGUMENT, "need n_layers, vocab (multiple of 8), hidden (multiple of 128) > 0");
    if (!w->embed || !w->final_norm || !w->lm_head || !w->layers) return fail(DT_ERR_INVALID_ARGUMENT, "null weights");
    for (int l = 0; l < w->n_layers; ++l) {
        const dt_model_layer_weights& L = w->layers[l];
        if (!L.q_proj || !L.k_proj || !L.v_proj || !L.o_proj || !L.q_norm || !L.k_norm || !L.post_attention_norm ||
            !L.gate_proj || !L.up_proj || !L.down_proj || !L.post_feedforward_norm)
            return fail(DT_ERR_INVALID_ARGUMENT, "null weight pointer in layer %d", l);
    }
    DeviceGuard dg;
    DT_TRY(dg.enter(device));
    int dev;
    DT_TRY(prepare_device(&dev));
    dt_model* m = new dt_model();
    m->device = device;
    m->n_layers = w->n_layers;
    m->vocab = w->vocab;
    m->d_model = w->d_model;
    m->n_heads = w->n_heads;
    m->hidden = w->hidden;
    m->eps = w->eps;
    m->theta = w->rope_theta;
    const int s = model_upload(m, w);
    if (s != DT_OK) {
        std::string msg = t_last_error;
        dt_model_destroy(m);
        t_last_error = msg;
        return s;
    }
    *out = m;
    return DT_OK;
}

int dt_model_create_from_npy(const char* folder, int n_layers, int device, dt_model** out) {
    t_last_error.clear();
    if (!folder || !out) return fail(DT_ERR_INVALID_ARGUMENT, "null argument");
    if (n_layers <= 0) n_layers = 16;
    const std::string f(folder);
    std::vector<std::vector<float>> store;
    store.reserve(3 + 11 * (size_t)n_layers);
    auto load = [&](const std::string& path, const float** dst, std::vector<long long>* shape_out) -> int {
        store.emplace_back();
        std::vector<long long> shape;
        DT_TRY(read_npy_f32(path, store.back(), shape));
        if (shape_out) *shape_out = shape;
        *dst = store.back().data();
        return DT_OK;
    };
    dt_model_weights w;
    std::vector<long long> es;
    DT_TRY(load(f + "/model.embed_tokens.weight.npy", &w.embed, &es));
    DT_TRY(load(f + "/model.norm.weight.npy", &w.final_norm, nullptr));
    std::vector<long long> ls;
    DT_TRY(load(f + "/lm_head.weight.npy", &w.lm_head, &ls));
    if (es.size() != 2 || ls.size() != 2 || es[1] != 2048 || ls[1] != 2048 || es[0] != ls[0])
        return fail(DT_ERR_IO, "embedding / lm_head shapes must be [vocab, 2048]");
    std::vector<dt_model_layer_weights> layers(n_layers);
    std::vector<long long> us;
    for (int l = 0; l < n_layers; ++l) {
        const std::string pre = f + "/model.layers." + std::to_string(l) + ".";
        dt_model_layer_weights& L = layers[l];
        DT_TRY(load(pre + "self_attn.q_proj.weight.npy", &L.q_proj, nullptr));
        DT_TRY(load(pre + "self_attn.k_proj.weight.npy", &L.k_proj, nullptr));
        DT_TRY(load(pre + "self_attn.v_proj.weight.npy", &L.v_proj, nullptr));
        DT_TRY(load(pre + "self_attn.o_proj.weight.npy", &L.o_proj, nullptr));
        DT_TRY(load(pre + "self_attn.q_norm.weight.npy", &L.q_norm, nullptr));
        DT_TRY(load(pre + "self_attn.k_norm.weight.npy", &L.k_norm, nullptr));
        DT_TRY(load(pre + "post_attention_layernorm.weight.npy", &L.post_attention_norm, nullptr));
        DT_TRY(load(pre + "mlp.gate_proj.weight.npy", &L.gate_proj, nullptr));
        DT_TRY(load(pre + "mlp.up_proj.weight.npy", &L.up_proj, &us));
        DT_TRY(load(pre + "mlp.down_proj.weight.npy", &L.down_proj, nullptr));
        DT_TRY(load(pre + "post_feedforward_layernorm.weight.npy", &L.post_feedforward_norm, nullptr));
    }
    w.layers = layers.data();
    w.n_layers = n_layers;
    w.vocab = (int)es[0];
    w.d_model = 2048;
    w.n_heads = 16;
    w.hidden = us.size() == 2 ? (int)us[0] : 8192;
    w.eps = 1e-6f;
    w.rope_theta = 500000.f;
    return dt_model_create(&w, device, out);
}

static size_t model_ws_bytes(const dt_model* m, long long M) {
    return 2 * align256(M * m->d_model * 4) + align256(M * m->d_model * 2) + attn_core_bytes(M) +
           align256(M * m->hidden * 2);
}

int dt_model_forward(dt_model* m, const uint32_t* tokens, int B, int T, float* logits, void* stream) {
    t_last_error.clear();
    if (!m) return fail(DT_ERR_INVALID_ARGUMENT, "null handle");
    if (B < 0 || T < 0) return fail(DT_ERR_INVALID_ARGUMENT, "negative shape");
    if (T > kMaxSeqLen) return fail(DT_ERR_INVALID_ARGUMENT, "T=%d exceeds max_seq_len %d", T, kMaxSeqLen);
    const long long M = (long long)B * T;
    if (M == 0) return DT_OK;
    if (!tokens || !logits || !aligned16(logits)) return fail(DT_ERR_INVALID_ARGUMENT, "tokens/logits invalid");
    DeviceGuard dg;
    DT_TRY(dg.enter(m->device));
    int dev;
    DT_TRY(prepare_device(&dev));
    const size_t need = model_ws_bytes(m, M);
    if (m->ws_bytes < need) {
        if (m->ws) DT_CUDA(cudaFree(m->ws));
        m->ws = nullptr;
        m->ws_bytes = 0;
        DT_CUDA(cudaMalloc(&m->ws, need));
        m->ws_bytes = need;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int d = m->d_model;
    uint8_t* w = reinterpret_cast<uint8_t*>(m->ws);
    float* x = reinterpret_cast<float*>(w);
    w += align256(M * d * 4);
    float* y = reinterpret_cast<float*>(w);
    w += align256(M * d * 4);
    __nv_bfloat16* xb = reinterpret_cast<__nv_bfloat16*>(w);
    w += align256(M * d * 2);
    uint8_t* attn_ws = w;
    w += attn_core_bytes(M);
    __nv_bfloat16* act = reinterpret_cast<__nv_bfloat16*>(w);
    const unsigned rows = (unsigned)M;
    dt::model::embed_gather_kernel<<<rows, dt::model::kThreads, 0, st>>>(tokens, m->embed, m->vocab, x, xb);
    DT_CUDA(cudaGetLastError());
    for (int l = 0; l < m->n_layers; ++l) {
        DT_TRY(attn_core(m->attn[l], xb, B, T, nullptr, y, attn_ws, dev, st));                  // attention
        dt::model::residual_norm_kernel<<<rows, dt::model::kThreads, 0, st>>>(x, y, m->pa_norm[l], x, xb, m->eps, 1);
        DT_CUDA(cudaGetLastError());                                                            // h = x + norm(attn)
        DT_TRY(launch_gemm(xb, m->w_gu[l], act, 1, (int)M, 2 * m->hidden, d, m->hidden, st, 1,
                           dt::gemm::kSwiGLU));                                                 // silu(g) * u
        DT_TRY(launch_gemm(act, m->w_down[l], y, 0, (int)M, d, m->hidden, d, st));             // down
        dt::model::residual_norm_kernel<<<rows, dt::model::kThreads, 0, st>>>(x, y, m->pf_norm[l], x, xb, m->eps, 1);
        DT_CUDA(cudaGetLastError());                                                            // x = h + norm(mlp)
    }
    dt::model::residual_norm_kernel<<<rows, dt::model::kThreads, 0, st>>>(nullptr, x, m->final_norm, nullptr, xb,
                                                                          m->eps, 0);          // final norm
    DT_CUDA(cudaGetLastError());
    return launch_gemm(xb, m->lm_head, logits, 0, (int)M, m->vocab, d, m->vocab, st);           // LM head
}

int dt_model_info(const dt_model* m, int* n_layers, int* vocab, int* hidden) {
    t_last_error.clear();
    if (!m) return fail(DT_ERR_INVALID_ARGUMENT, "null handle");
    if (n_layers) *n_layers = m->n_layers;
    if (vocab) *vocab = m->vocab;
    if (hidden) *hidden = m->hidden;
    return DT_OK;
}

int dt_model_forward_host(dt_model* m, const uint32_t* tokens, int B, int T, float* logits) {
    t_last_error.clear();
    if (!m) return fail(DT_ERR_INVALID_ARGUMENT, "null handle");
    if (B < 0 || T < 0) return fail(DT_ERR_INVALID_ARGUMENT, "negative shape");
    const long long M = (long long)B * T;
    if (M == 0) return DT_OK;
    if (!tokens || !logits) return fail(DT_ERR_INVALID_ARGUMENT, "null tokens/logits");
    for (long long i = 0; i < M; ++i)
        if (tokens[i] >= (uint32_t)m->vocab)
            return fail(DT_ERR_INVALID_ARGUMENT, "token id %u at position %lld is not below the vocabulary size %d",
                        tokens[i], i, m->vocab);
    DeviceGuard dg;
    DT_TRY(dg.enter(m->device));
    if (!m->stream) DT_CUDA(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    const size_t lb = align256((size_t)M * m->vocab * 4);
    const size_t need = lb + align256((size_t)M * 4);
    if (m->io_bytes < need) {
        if (m->io) DT_CUDA(cudaFree(m->io));
        m->io = nullptr;
        m->io_bytes = 0;
        DT_CUDA(cudaMalloc(&m->io, need));
        m->io_bytes = need;
    }
    float* dl = reinterpret_cast<float*>(m->io);
    uint32_t* dt_ids = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(m->io) + lb);
    DT_CUDA(cudaMemcpyAsync(dt_ids, tokens, (size_t)M * 4, cudaMemcpyHostToDevice, m->stream));
    DT_TRY(dt_model_forward(m, dt_ids, B, T, dl, m->stream));
    DT_CUDA(cudaMemcpyAsync(logits, dl, (size_t)M * m->vocab * 4, cudaMemcpyDeviceToHost, m->stream));
    DT_CUDA(cudaStreamSynchronize(m->stream));
    bool had;
    return read_device_error(&had);
}

}  // extern "C"
