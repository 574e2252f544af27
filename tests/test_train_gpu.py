"""GPU parity of the attention layer's training path (OlmoAttention::backward,
step, zero_grad; OlmoAttention.cpp:189-330, RMSNorm.cpp:24-41) through the C
ABI, against the oracle's restatement (pinned to fp64 autograd on the CPU)."""
import numpy as np
import pytest

import oracle
from common import TOL_LAYER_BWD_REL_L2, layer_weights, randn, rel_l2

pytestmark = pytest.mark.gpu

KEYS = ("q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm")


def _layer(ws):
    import dirktensor_b200 as dt

    return dt.OlmoAttention.from_weights(*ws)


@pytest.mark.parametrize("B,T", [(1, 128), (2, 200), (1, 520)])
def test_layer_backward_vs_oracle(cuda, B, T):
    import torch

    import dirktensor_b200 as dt

    ws = layer_weights(60 + T)
    x = randn(61 + T, (B, T, 2048))
    dy = randn(62 + T, (B, T, 2048))
    attn = _layer(ws)
    attn.forward(torch.from_numpy(x).to(cuda))
    dx = attn.backward(torch.from_numpy(dy).to(cuda)).cpu().numpy()
    grads = attn.parameters(gradients=True)
    dt.check_device_error()
    _, saved = oracle.attention_layer_train(x, *ws)
    rdx, rg = oracle.attention_layer_backward(dy, saved, *ws)
    assert rel_l2(dx, rdx) < TOL_LAYER_BWD_REL_L2, rel_l2(dx, rdx)
    for k in KEYS:
        assert rel_l2(grads[k], rg[k]) < TOL_LAYER_BWD_REL_L2, (k, rel_l2(grads[k], rg[k]))
    attn.close()


def test_gradients_accumulate_zero_grad_and_step(cuda):
    import torch

    import dirktensor_b200 as dt

    ws = layer_weights(70)
    B, T = 1, 160
    x = torch.from_numpy(randn(71, (B, T, 2048))).to(cuda)
    dy = torch.from_numpy(randn(72, (B, T, 2048))).to(cuda)
    attn = _layer(ws)
    attn.forward(x)
    attn.backward(dy)
    g1 = attn.parameters(gradients=True)
    attn.forward(x)
    attn.backward(dy)
    g2 = attn.parameters(gradients=True)
    for k in KEYS:  # the reference accumulates (beta = 1) until zero_grad
        assert rel_l2(g2[k], 2 * g1[k]) < 1e-5, k
    attn.zero_grad()
    g0 = attn.parameters(gradients=True)
    assert all(not np.any(g0[k]) for k in KEYS)
    # one step: w -= lr * grad on the fp32 master weights
    attn.forward(x)
    attn.backward(dy)
    g = attn.parameters(gradients=True)
    before = attn.parameters()
    lr = 1e-3
    attn.step(lr)
    after = attn.parameters()
    dt.check_device_error()
    for k in KEYS:
        assert np.allclose(after[k], before[k] - np.float32(lr) * g[k], rtol=0, atol=1e-6), k
    # the next forward uses the updated weights
    y = attn.forward(x).cpu().numpy()
    ref = oracle.attention_layer(x.cpu().numpy(), *(after[k] for k in KEYS))
    assert rel_l2(y, ref) < 1.5e-2
    attn.close()


def test_host_api_matches_device_api(cuda):
    import torch

    ws = layer_weights(80)
    x = randn(81, (1, 96, 2048))
    dy = randn(82, (1, 96, 2048))
    a1, a2 = _layer(ws), _layer(ws)
    a1.forward(x)
    dx_h = a1.backward(dy)
    a2.forward(torch.from_numpy(x).to(cuda))
    dx_d = a2.backward(torch.from_numpy(dy).to(cuda)).cpu().numpy()
    assert np.array_equal(dx_h, dx_d)
    g1, g2 = a1.parameters(gradients=True), a2.parameters(gradients=True)
    assert all(np.array_equal(g1[k], g2[k]) for k in KEYS)
    a1.close()
    a2.close()


def test_backward_rejects_shape_mismatch_and_varlen(cuda):
    import torch

    import dirktensor_b200 as dt

    attn = _layer(layer_weights(90))
    x = torch.from_numpy(randn(91, (2, 128, 2048))).to(cuda)
    attn.forward(x)
    with pytest.raises(dt.DTError):
        attn.backward(torch.zeros((1, 128, 2048), device=cuda))
    attn.forward(x, seq_lens=[100, 128])
    with pytest.raises(dt.DTError):
        attn.backward(torch.zeros((2, 128, 2048), device=cuda))
    attn.close()
