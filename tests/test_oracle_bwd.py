"""CPU tests: the oracle's training-path restatements pinned to the reference.

Pins: golden vectors from the reference's own flash_attention_backward
(tests/golden/flash_bwd_ref.npz), the live reference library when it was built
here, an fp64 truth of the attention gradients, and torch fp64 autograd of the
whole layer (OlmoAttention.cpp's backward cannot be compiled here: it needs far
more of xtensor than the shims provide)."""
import os

import numpy as np
import pytest
import torch

import oracle
from common import SCALE, layer_weights, qkv, randn, rel_l2

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "flash_bwd_ref.npz")


def _checksum(*arrs):
    return float(sum(np.sum(a.astype(np.float64) * (1 + np.arange(a.size).reshape(a.shape) % 7)) for a in arrs))


def _cases():
    z = np.load(GOLDEN)
    return sorted({k.split("__")[0] for k in z.files})


@pytest.mark.parametrize("name", _cases())
def test_oracle_flash_bwd_matches_reference_golden(name):
    z = np.load(GOLDEN)
    seed, B, T, H, causal = (int(x) for x in z[f"{name}__meta"])
    q, k, v = qkv(seed, B, T, H)
    do = randn(seed + 1000, q.shape)
    assert _checksum(q, k, v, do) == pytest.approx(float(z[f"{name}__checksum"][0]), rel=1e-12)
    o, m, l = oracle.flash_fwd(q, k, v, SCALE, bool(causal))
    dq, dk, dv = oracle.flash_bwd(do, o, m, l, q, k, v, SCALE, bool(causal))
    for got, key in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
        ref = z[f"{name}__{key}"]
        assert np.max(np.abs(got - ref)) < 2e-5 * max(1.0, float(np.max(np.abs(ref)))), key


def _attn_grads_f64(q, k, v, do, scale, causal):
    """fp64 truth: P = softmax(scale QK^T + mask), O = PV; the gradients of <O, dO>."""
    q, k, v, do = (torch.from_numpy(a.astype(np.float64)).permute(0, 2, 1, 3).requires_grad_(True)
                   for a in (q, k, v, do))
    T = q.shape[2]
    s = scale * q @ k.transpose(-1, -2)
    if causal:
        s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), float("-inf"))
    o = torch.softmax(s, -1) @ v
    (o * do.detach()).sum().backward()
    return [t.grad.permute(0, 2, 1, 3).numpy() for t in (q, k, v)]


@pytest.mark.parametrize("B,T,H,causal", [(1, 200, 2, True), (2, 70, 1, True), (1, 130, 2, False)])
def test_oracle_flash_bwd_matches_fp64_truth(B, T, H, causal):
    q, k, v = qkv(40 + T, B, T, H)
    do = randn(41 + T, q.shape)
    o, m, l = oracle.flash_fwd(q, k, v, SCALE, causal)
    got = oracle.flash_bwd(do, o, m, l, q, k, v, SCALE, causal)
    for g, t in zip(got, _attn_grads_f64(q, k, v, do, SCALE, causal)):
        assert rel_l2(g, t) < 1e-5


@pytest.mark.skipif(oracle.ref_lib() is None, reason="reference library not built (no reference sources)")
def test_oracle_flash_bwd_matches_reference_library_live():
    q, k, v = qkv(6, 2, 520, 2)
    do = randn(7, q.shape)
    o, m, l, _ = oracle.ref_flash_fwd(q, k, v, SCALE, True)
    got = oracle.flash_bwd(do, o, m, l, q, k, v, SCALE, True)
    ref = oracle.ref_flash_bwd(do, o, m, l, q, k, v, SCALE, True)[:3]
    for g, r in zip(got, ref):
        assert np.max(np.abs(g - r)) < 2e-5 * max(1.0, float(np.max(np.abs(r))))


def test_rope_bwd_is_the_adjoint_of_rope():
    x = randn(1, (2, 9, 4, 128))
    y = randn(2, (2, 9, 4, 128))
    s, c = oracle.rope_tables(9)
    lhs = np.sum(oracle.rope(x, s, c).astype(np.float64) * y)
    rhs = np.sum(x.astype(np.float64) * oracle.rope_bwd(y, s, c))
    assert abs(lhs - rhs) < 1e-4 * abs(lhs) + 1e-3


def test_rmsnorm_bwd_matches_fp64_autograd():
    x = randn(3, (5, 2048))
    g = (1 + randn(4, (2048,), 0.02)).astype(np.float32)
    dy = randn(5, (5, 2048))
    y, rms = oracle.rmsnorm_rms(x, g)
    dx, dg = oracle.rmsnorm_bwd(dy, y, g, rms)
    xt = torch.from_numpy(x.astype(np.float64)).requires_grad_(True)
    gt = torch.from_numpy(g.astype(np.float64)).requires_grad_(True)
    yt = xt / torch.sqrt((xt ** 2).mean(-1, keepdim=True) + 1e-6) * gt
    (yt * torch.from_numpy(dy.astype(np.float64))).sum().backward()
    assert rel_l2(dx, xt.grad.numpy()) < 1e-5
    assert rel_l2(dg, gt.grad.numpy()) < 1e-5


def _layer_autograd_f64(x, ws, dy, n_heads=16):
    """torch fp64 autograd of OlmoAttention::forward (OlmoAttention.cpp:56-108)."""
    wq, wk, wv, wo, qg, kg = (torch.from_numpy(w.astype(np.float64)).requires_grad_(True) for w in ws)
    xt = torch.from_numpy(x.astype(np.float64)).requires_grad_(True)
    B, T, d = x.shape
    hd = d // n_heads

    def norm(a, gain):
        return a / torch.sqrt((a ** 2).mean(-1, keepdim=True) + 1e-6) * gain

    s_t, c_t = oracle.rope_tables(T, hd)
    s_t, c_t = torch.from_numpy(s_t.astype(np.float64)), torch.from_numpy(c_t.astype(np.float64))

    def rope(a):
        a = a.view(B, T, n_heads, hd)
        a1, a2 = a[..., :hd // 2], a[..., hd // 2:]
        cs, sn = c_t[None, :, None, :], s_t[None, :, None, :]
        return torch.cat([a1 * cs[..., :hd // 2] - a2 * sn[..., :hd // 2],
                          a2 * cs[..., hd // 2:] + a1 * sn[..., hd // 2:]], -1)

    q = rope(norm(xt @ wq.T, qg)).permute(0, 2, 1, 3)
    k = rope(norm(xt @ wk.T, kg)).permute(0, 2, 1, 3)
    v = (xt @ wv.T).view(B, T, n_heads, hd).permute(0, 2, 1, 3)
    s = (q @ k.transpose(-1, -2)) / np.sqrt(hd)
    s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), float("-inf"))
    a = (torch.softmax(s, -1) @ v).permute(0, 2, 1, 3).reshape(B, T, d)
    y = a @ wo.T
    (y * torch.from_numpy(dy.astype(np.float64))).sum().backward()
    return xt.grad.numpy(), [w.grad.numpy() for w in (wq, wk, wv, wo, qg, kg)]


def test_layer_backward_matches_fp64_autograd():
    ws = layer_weights(50)
    B, T = 2, 40
    x = randn(51, (B, T, 2048))
    dy = randn(52, (B, T, 2048))
    y, saved = oracle.attention_layer_train(x, *ws)
    assert rel_l2(y, oracle.attention_layer(x, *ws)) < 1e-6
    dx, g = oracle.attention_layer_backward(dy, saved, *ws)
    tdx, tg = _layer_autograd_f64(x, ws, dy)
    assert rel_l2(dx, tdx) < 1e-4
    for key, t in zip(("q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm"), tg):
        assert rel_l2(g[key], t) < 1e-4, key
