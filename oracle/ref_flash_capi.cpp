// TEST INFRASTRUCTURE (oracle) -- not part of the product.
//
// C entry points around the reference's own flash_attention_forward
// (FlashAttention.cpp:24-182, declared FlashAttention.h:15-21) and
// flash_attention_backward (FlashAttention.cpp:185-359, FlashAttention.h:33-43), compiled in
// place from the reference tree against the shims in oracle/shims.  Used to
// pin the C restatement in oracle.c and as the timed CPU baseline.  Only
// tests/, the smoke check and bench.py's CPU-baseline legs load it.
#include <chrono>
#include <cstring>
#include <thread>

#include "FlashAttention.h"
#include "cblas.h"

static int g_threads = 0;

int ref_shim_threads() {
    if (g_threads > 0) return g_threads;
    const unsigned hc = std::thread::hardware_concurrency();
    return hc ? static_cast<int>(hc) : 1;
}

extern "C" {

// Number of host threads the TBB shim uses (0 = all cores).
void ref_set_threads(int n) { g_threads = n; }

int ref_get_threads(void) { return ref_shim_threads(); }

// Runs the reference's flash_attention_forward on [B,T,H,D] fp32 host arrays.
// o: [B,T,H,D]; m, l: [B,T,H] (may be null).  Returns the wall time of the
// flash_attention_forward call alone in seconds (input copies into the
// container are excluded), or a negative value on error.
double ref_flash_forward(const float* q, const float* k, const float* v, float* o, float* m, float* l,
                         long B, long T, long H, long D, float scale, int causal) {
    try {
        const std::array<std::size_t, 4> s4{(size_t)B, (size_t)T, (size_t)H, (size_t)D};
        xt::xtensor<float, 4> Q(s4), K(s4), V(s4);
        const size_t n = (size_t)B * T * H * D;
        std::memcpy(Q.data(), q, n * sizeof(float));
        std::memcpy(K.data(), k, n * sizeof(float));
        std::memcpy(V.data(), v, n * sizeof(float));
        // The reference nests BLAS calls inside its (batch, head) parallel loop:
        // keep BLAS single-threaded there so the shim's threads are the parallelism.
        scipy_openblas_set_num_threads(1);
        const auto t0 = std::chrono::steady_clock::now();
        FlashAttentionResult r = flash_attention_forward(Q, K, V, scale, causal != 0);
        const auto t1 = std::chrono::steady_clock::now();
        std::memcpy(o, r.output.data(), n * sizeof(float));
        const size_t ns = (size_t)B * T * H;
        if (m) std::memcpy(m, r.softmax_m.data(), ns * sizeof(float));
        if (l) std::memcpy(l, r.softmax_l.data(), ns * sizeof(float));
        return std::chrono::duration<double>(t1 - t0).count();
    } catch (...) {
        return -1.0;
    }
}

// Runs the reference's flash_attention_backward on [B,T,H,D] fp32 host arrays
// (m, l: [B,T,H]).  Returns the wall time of the call in seconds, or a negative
// value on error.
double ref_flash_backward(const float* dout, const float* out, const float* m, const float* l, const float* q,
                          const float* k, const float* v, float* dq, float* dk, float* dv, long B, long T, long H,
                          long D, float scale, int causal) {
    try {
        const std::array<std::size_t, 4> s4{(size_t)B, (size_t)T, (size_t)H, (size_t)D};
        const std::array<std::size_t, 3> s3{(size_t)B, (size_t)T, (size_t)H};
        xt::xtensor<float, 4> dO(s4), O(s4), Q(s4), K(s4), V(s4);
        xt::xtensor<float, 3> M(s3), L(s3);
        const size_t n = (size_t)B * T * H * D, ns = (size_t)B * T * H;
        std::memcpy(dO.data(), dout, n * sizeof(float));
        std::memcpy(O.data(), out, n * sizeof(float));
        std::memcpy(Q.data(), q, n * sizeof(float));
        std::memcpy(K.data(), k, n * sizeof(float));
        std::memcpy(V.data(), v, n * sizeof(float));
        std::memcpy(M.data(), m, ns * sizeof(float));
        std::memcpy(L.data(), l, ns * sizeof(float));
        scipy_openblas_set_num_threads(1);
        const auto t0 = std::chrono::steady_clock::now();
        FlashAttentionGradients g = flash_attention_backward(dO, O, M, L, Q, K, V, scale, causal != 0);
        const auto t1 = std::chrono::steady_clock::now();
        std::memcpy(dq, g.d_Q.data(), n * sizeof(float));
        std::memcpy(dk, g.d_K.data(), n * sizeof(float));
        std::memcpy(dv, g.d_V.data(), n * sizeof(float));
        return std::chrono::duration<double>(t1 - t0).count();
    } catch (...) {
        return -1.0;
    }
}

}  // extern "C"
