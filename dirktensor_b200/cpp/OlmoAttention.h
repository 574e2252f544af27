// Drop-in for the reference's OlmoAttention (OlmoAttention.h:10-42): the same
// public interface, so OlmoBlock (which holds it by value, OlmoBlock.h:19, and
// calls forward/backward/step/zero_grad, OlmoBlock.cpp:6-40) compiles
// unchanged.  The weights live on the GPU (bf16 projections, fp32 norm gains)
// behind an opaque handle of the C ABI (with the fp32 master weights and
// gradients of the training path); the class is therefore move-only.
#pragma once

#include <string>
#include <xtensor/containers/xtensor.hpp>

struct dt_attn;
struct dt_comm;

namespace dirktensor_b200 {
// Head-parallel mode for this process (one process, or thread, per GPU of one
// node; comm from dt_comm_create).  After set_tensor_parallel(comm), every
// OlmoAttention constructed from (folder, index) holds only this rank's heads
// of the layer (dt_attn_create_sharded_from_npy), and forward() returns the
// whole [batch, seq, d_model] output on every rank (the ranks' token slices
// all-gathered), so OlmoBlock and OlmoModel run head-parallel unchanged; every
// rank must call forward with the same input.  exchange: 0 = the attention
// kernel stores rows into their owners' buffers over NVLink, 1 = NCCL
// all-to-all.  backward/step/zero_grad stay single-GPU and throw on a
// head-parallel layer.  set_tensor_parallel(nullptr) returns to one GPU for
// layers constructed afterwards; the communicator must outlive the layers.
void set_tensor_parallel(dt_comm* comm, int exchange = 0);
}  // namespace dirktensor_b200

class OlmoAttention {
public:
    // Loads {folder}/model.layers.{index}.self_attn.{q,k,v,o}_proj.weight.npy and
    // {q,k}_norm.weight.npy (OlmoAttention.cpp:39-46).  The GPU is taken from
    // the DIRKTENSOR_B200_DEVICE environment variable (default 0).
    OlmoAttention(const std::string& folder, unsigned int index);
    ~OlmoAttention();
    OlmoAttention(OlmoAttention&& other) noexcept;
    OlmoAttention& operator=(OlmoAttention&& other) noexcept;
    OlmoAttention(const OlmoAttention&) = delete;
    OlmoAttention& operator=(const OlmoAttention&) = delete;

    // input (batch, seq, d_model) -> (batch, seq, d_model)  (OlmoAttention.cpp:56-108)
    xt::xtensor<float, 3> forward(const xt::xtensor<float, 3>& input);
    // Gradient of the last forward's input (OlmoAttention.cpp:189-312); the
    // weight gradients accumulate on the GPU until zero_grad().
    xt::xtensor<float, 3> backward(const xt::xtensor<float, 3>& d_output);
    // w -= lr * grad for every parameter (OlmoAttention.cpp:315-322).
    void step(float lr);
    // Clears the accumulated gradients (OlmoAttention.cpp:324-330).
    void zero_grad();

private:
    dt_attn* m_handle = nullptr;
    bool m_sharded = false;
};
