// OlmoModel over the C ABI (dt_model_create_from_npy / dt_model_forward_host).
#include "OlmoModel.h"

#include <cstdlib>
#include <stdexcept>
#include <string>
#include <utility>

#include "dirktensor_b200.h"
#include "model_config.h"

OlmoModel::OlmoModel(const std::string& folder, unsigned int layers) {
    const char* s = std::getenv("DIRKTENSOR_B200_DEVICE");
    const int device = s ? std::atoi(s) : 0;
    const int count = static_cast<int>(layers ? layers : n_layers);
    if (dt_model_create_from_npy(folder.c_str(), count, device, &m_handle) != DT_OK)
        throw std::runtime_error(std::string("OlmoModel: ") + dt_last_error());
    dt_model_info(m_handle, nullptr, &m_vocab, nullptr);
}

OlmoModel::~OlmoModel() {
    if (m_handle) dt_model_destroy(m_handle);
}

OlmoModel::OlmoModel(OlmoModel&& other) noexcept
    : m_handle(std::exchange(other.m_handle, nullptr)), m_vocab(other.m_vocab) {}

OlmoModel& OlmoModel::operator=(OlmoModel&& other) noexcept {
    if (this != &other) {
        if (m_handle) dt_model_destroy(m_handle);
        m_handle = std::exchange(other.m_handle, nullptr);
        m_vocab = other.m_vocab;
    }
    return *this;
}

xt::xtensor<float, 3> OlmoModel::forward(const xt::xtensor<uint32_t, 2>& batch) {
    const std::size_t b = batch.shape(0), t = batch.shape(1);
    xt::xtensor<float, 3> logits = xt::empty<float>({b, t, static_cast<std::size_t>(m_vocab)});
    if (dt_model_forward_host(m_handle, batch.data(), static_cast<int>(b), static_cast<int>(t), logits.data()) != DT_OK)
        throw std::runtime_error(std::string("OlmoModel::forward: ") + dt_last_error());
    return logits;
}

void OlmoModel::backward(const xt::xtensor<float, 3>&) {
    throw std::logic_error("OlmoModel::backward: the B200 drop-in implements the forward path only");
}

void OlmoModel::step(float) {
    throw std::logic_error("OlmoModel::step: the B200 drop-in implements the forward path only");
}

void OlmoModel::zero_grad() {}
