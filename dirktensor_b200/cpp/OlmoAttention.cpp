// OlmoAttention over the C ABI (dt_attn_create_from_npy, dt_attn_forward_host,
// dt_attn_backward_host, dt_attn_step, dt_attn_zero_grad; head-parallel:
// dt_attn_create_sharded_from_npy, dt_attn_forward_sharded_host).
#include "OlmoAttention.h"

#include <cstdlib>
#include <stdexcept>
#include <string>
#include <utility>

#include "dirktensor_b200.h"
#include "model_config.h"

namespace {
int device_from_env() {
    const char* s = std::getenv("DIRKTENSOR_B200_DEVICE");
    return s ? std::atoi(s) : 0;
}
[[noreturn]] void raise(const char* what) { throw std::runtime_error(std::string(what) + ": " + dt_last_error()); }
dt_comm* g_tp_comm = nullptr;
int g_tp_exchange = 0;
}  // namespace

void dirktensor_b200::set_tensor_parallel(dt_comm* comm, int exchange) {
    g_tp_comm = comm;
    g_tp_exchange = exchange;
}

OlmoAttention::OlmoAttention(const std::string& folder, unsigned int index) {
    if (g_tp_comm) {
        if (dt_attn_create_sharded_from_npy(folder.c_str(), index, g_tp_comm, g_tp_exchange, &m_handle) != DT_OK)
            raise("OlmoAttention");
        m_sharded = true;
    } else if (dt_attn_create_from_npy(folder.c_str(), index, device_from_env(), &m_handle) != DT_OK) {
        raise("OlmoAttention");
    }
}

OlmoAttention::~OlmoAttention() {
    if (m_handle) dt_attn_destroy(m_handle);
}

OlmoAttention::OlmoAttention(OlmoAttention&& other) noexcept
    : m_handle(std::exchange(other.m_handle, nullptr)), m_sharded(other.m_sharded) {}

OlmoAttention& OlmoAttention::operator=(OlmoAttention&& other) noexcept {
    if (this != &other) {
        if (m_handle) dt_attn_destroy(m_handle);
        m_handle = std::exchange(other.m_handle, nullptr);
        m_sharded = other.m_sharded;
    }
    return *this;
}

xt::xtensor<float, 3> OlmoAttention::forward(const xt::xtensor<float, 3>& input) {
    const std::size_t b = input.shape(0), t = input.shape(1), d = input.shape(2);
    if (d != d_model) throw std::invalid_argument("OlmoAttention::forward: last dimension must be d_model");
    xt::xtensor<float, 3> out = xt::empty<float>({b, t, d});
    const int st = m_sharded ? dt_attn_forward_sharded_host(m_handle, input.data(), static_cast<int>(b),
                                                             static_cast<int>(t), nullptr, 1, out.data())
                             : dt_attn_forward_host(m_handle, input.data(), static_cast<int>(b), static_cast<int>(t),
                                                    nullptr, out.data());
    if (st != DT_OK) raise("OlmoAttention::forward");
    return out;
}

xt::xtensor<float, 3> OlmoAttention::backward(const xt::xtensor<float, 3>& d_output) {
    const std::size_t b = d_output.shape(0), t = d_output.shape(1), d = d_output.shape(2);
    if (d != d_model) throw std::invalid_argument("OlmoAttention::backward: last dimension must be d_model");
    xt::xtensor<float, 3> d_input = xt::empty<float>({b, t, d});
    if (dt_attn_backward_host(m_handle, d_output.data(), static_cast<int>(b), static_cast<int>(t),
                              d_input.data()) != DT_OK)
        raise("OlmoAttention::backward");
    return d_input;
}

void OlmoAttention::step(float lr) {
    if (dt_attn_step(m_handle, lr, nullptr) != DT_OK) raise("OlmoAttention::step");
}

void OlmoAttention::zero_grad() {
    if (dt_attn_zero_grad(m_handle, nullptr) != DT_OK) raise("OlmoAttention::zero_grad");
}
