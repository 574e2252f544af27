// flash_attention_forward over the C ABI (dt_flash_fwd_host).
#include "FlashAttention.h"

#include <stdexcept>
#include <string>

#include "dirktensor_b200.h"

FlashAttentionResult flash_attention_forward(const xt::xtensor<float, 4>& Q, const xt::xtensor<float, 4>& K,
                                             const xt::xtensor<float, 4>& V, float scale, bool causal) {
    const std::size_t b = Q.shape(0), t = Q.shape(1), h = Q.shape(2), d = Q.shape(3);
    for (const auto* x : {&K, &V})
        if (x->shape(0) != b || x->shape(1) != t || x->shape(2) != h || x->shape(3) != d)
            throw std::invalid_argument("flash_attention_forward: Q, K, V shapes differ");
    FlashAttentionResult r;
    r.output = xt::empty<float>({b, t, h, d});
    r.softmax_m = xt::empty<float>({b, t, h});
    r.softmax_l = xt::empty<float>({b, t, h});
    const int st = dt_flash_fwd_host(Q.data(), K.data(), V.data(), r.output.data(), r.softmax_m.data(),
                                     r.softmax_l.data(), static_cast<int>(b), static_cast<int>(t),
                                     static_cast<int>(h), static_cast<int>(d), scale, causal ? 1 : 0);
    if (st != DT_OK) throw std::runtime_error(std::string("flash_attention_forward: ") + dt_last_error());
    return r;
}

FlashAttentionGradients flash_attention_backward(const xt::xtensor<float, 4>& d_output,
                                                 const xt::xtensor<float, 4>& output,
                                                 const xt::xtensor<float, 3>& softmax_m,
                                                 const xt::xtensor<float, 3>& softmax_l,
                                                 const xt::xtensor<float, 4>& Q, const xt::xtensor<float, 4>& K,
                                                 const xt::xtensor<float, 4>& V, float scale, bool causal) {
    const std::size_t b = Q.shape(0), t = Q.shape(1), h = Q.shape(2), d = Q.shape(3);
    for (const auto* x : {&d_output, &output, &K, &V})
        if (x->shape() != Q.shape())
            throw std::invalid_argument("flash_attention_backward: d_output, output, Q, K, V shapes differ");
    for (const auto* s : {&softmax_m, &softmax_l})
        if (s->shape(0) != b || s->shape(1) != t || s->shape(2) != h)
            throw std::invalid_argument("flash_attention_backward: softmax_m and softmax_l must be (batch, seq, n_heads)");
    FlashAttentionGradients g;
    g.d_Q = xt::empty<float>({b, t, h, d});
    g.d_K = xt::empty<float>({b, t, h, d});
    g.d_V = xt::empty<float>({b, t, h, d});
    if (dt_flash_bwd_host(d_output.data(), output.data(), softmax_m.data(), softmax_l.data(), Q.data(), K.data(),
                          V.data(), g.d_Q.data(), g.d_K.data(), g.d_V.data(), static_cast<int>(b),
                          static_cast<int>(t), static_cast<int>(h), static_cast<int>(d), scale, causal ? 1 : 0) != DT_OK)
        throw std::runtime_error(std::string("flash_attention_backward: ") + dt_last_error());
    return g;
}
