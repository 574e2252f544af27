// Drop-in for the reference's OlmoModel (OlmoModel.h:11-31): the same public
// interface -- constructed from a checkpoint folder, forward on a batch of
// uint32 token ids returning logits (batch, seq, vocab) -- with the whole
// prefill (embedding, 16 decoder layers, final norm, LM head) on the GPU
// through the C ABI in include/dirktensor_b200.h.  Move-only (owns a device
// handle).  The training path (backward, step) is not provided.
#pragma once

#include <cstdint>
#include <string>
#include <xtensor/containers/xtensor.hpp>

struct dt_model;

class OlmoModel {
public:
    // Reads {folder}/model.embed_tokens.weight.npy, model.norm.weight.npy,
    // lm_head.weight.npy and the per-layer files (OlmoModel.cpp:11-22).  The GPU
    // is taken from DIRKTENSOR_B200_DEVICE (default 0).  `layers` defaults to
    // model_config.h's n_layers (16); a smaller value loads only the first layers.
    explicit OlmoModel(const std::string& folder, unsigned int layers = 0);
    ~OlmoModel();
    OlmoModel(OlmoModel&& other) noexcept;
    OlmoModel& operator=(OlmoModel&& other) noexcept;
    OlmoModel(const OlmoModel&) = delete;
    OlmoModel& operator=(const OlmoModel&) = delete;

    // batch (batch, seq) token ids -> logits (batch, seq, vocab)  (OlmoModel.cpp:25-48)
    xt::xtensor<float, 3> forward(const xt::xtensor<uint32_t, 2>& batch);
    // Training path (OlmoModel.cpp:50-83): not provided; throws std::logic_error.
    void backward(const xt::xtensor<float, 3>& d_output);
    void step(float lr);
    void zero_grad();

private:
    dt_model* m_handle = nullptr;
    int m_vocab = 0;
};
