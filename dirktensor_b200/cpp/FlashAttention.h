// Drop-in for the reference's FlashAttention.h (FlashAttention.h:1-43): the
// same types and function signatures, computed on a B200 through the C ABI in
// include/dirktensor_b200.h.  Tensors are host xt::xtensor (row-major), copied
// to the device and back inside each call.
#pragma once

#include <xtensor/containers/xtensor.hpp>

// Result with the statistics a backward pass would need (FlashAttention.h:6-10).
struct FlashAttentionResult {
    xt::xtensor<float, 4> output;     // (batch, seq, n_heads, head_dim)
    xt::xtensor<float, 3> softmax_m;  // (batch, seq, n_heads): row max of the scaled scores
    xt::xtensor<float, 3> softmax_l;  // (batch, seq, n_heads): sum of exp(score - max)
};

// Causal (or full) attention forward (FlashAttention.h:15-21).  Q, K, V:
// (batch, seq, n_heads, head_dim) with head_dim 128.  Throws std::runtime_error
// with the library's message on failure.
FlashAttentionResult flash_attention_forward(const xt::xtensor<float, 4>& Q, const xt::xtensor<float, 4>& K,
                                             const xt::xtensor<float, 4>& V, float scale, bool causal = true);

// Gradients of the backward pass (FlashAttention.h:27-31).
struct FlashAttentionGradients {
    xt::xtensor<float, 4> d_Q;
    xt::xtensor<float, 4> d_K;
    xt::xtensor<float, 4> d_V;
};

// Attention backward (FlashAttention.h:33-43): dQ, dK, dV from the upstream
// gradient, the forward output and its statistics.  Throws std::runtime_error
// with the library's message on failure.
FlashAttentionGradients flash_attention_backward(const xt::xtensor<float, 4>& d_output,
                                                 const xt::xtensor<float, 4>& output,
                                                 const xt::xtensor<float, 3>& softmax_m,
                                                 const xt::xtensor<float, 3>& softmax_l,
                                                 const xt::xtensor<float, 4>& Q, const xt::xtensor<float, 4>& K,
                                                 const xt::xtensor<float, 4>& V, float scale, bool causal = true);
