"""GPU parity of the attention backward (flash_attention_backward,
FlashAttention.cpp:185-359) through the C ABI.

Compares dQ, dK, dV against the oracle's restatement (itself pinned to the
reference's own backward), against the reference's golden vectors, and at the
configuration sizes against torch fp32 autograd of the same attention on the
GPU.  Tolerance (bf16 tensor-core operands; fp32 softmax and accumulation) in
tests/common.py."""
import os

import numpy as np
import pytest

import oracle
from common import SCALE, TOL_BWD_REL_L2, qkv, randn

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "flash_bwd_ref.npz")


def dt_bwd(cuda, do, o, m, l, q, k, v, causal=True):
    import torch

    import dirktensor_b200 as dt

    args = [torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for a in (do, o, m, l, q, k, v)]
    g = dt.flash_attention_backward(*args, SCALE, causal)
    dt.check_device_error()
    return [t.cpu().numpy() for t in g]


def check(got, ref, tag=""):
    """Relative L2 error of each gradient.  dQ and dK can vanish exactly (T = 1:
    P = 1 and dP = D, so dS = 0); their error is then measured against the
    scale of dV, the gradient that keeps the magnitude of dO."""
    scale_dv = float(np.linalg.norm(np.asarray(ref[2], np.float64)))
    for g, r, n in zip(got, ref, ("dq", "dk", "dv")):
        r64 = np.asarray(r, np.float64)
        err = float(np.linalg.norm(np.asarray(g, np.float64) - r64) / max(np.linalg.norm(r64), scale_dv, 1e-30))
        assert err < TOL_BWD_REL_L2, (tag, n, err)
        assert np.all(np.isfinite(g)), (tag, n)


@pytest.mark.parametrize("B,T,H,causal", [(1, 1, 2, True), (1, 63, 2, True), (2, 129, 1, True), (1, 256, 2, True),
                                          (1, 300, 3, True), (2, 520, 2, True), (1, 300, 1, False),
                                          (1, 1000, 4, True)])
def test_flash_bwd_vs_oracle(cuda, B, T, H, causal):
    q, k, v = qkv(3000 + T + B, B, T, H)
    do = randn(3100 + T, q.shape)
    o, m, l = oracle.flash_fwd(q, k, v, SCALE, causal)
    got = dt_bwd(cuda, do, o, m, l, q, k, v, causal)
    check(got, oracle.flash_bwd(do, o, m, l, q, k, v, SCALE, causal), (B, T, H, causal))


def test_flash_bwd_vs_reference_golden(cuda):
    z = np.load(GOLDEN)
    names = sorted({k.split("__")[0] for k in z.files})
    assert names
    for name in names:
        seed, B, T, H, causal = (int(x) for x in z[f"{name}__meta"])
        q, k, v = qkv(seed, B, T, H)
        do = randn(seed + 1000, q.shape)
        o, m, l = oracle.flash_fwd(q, k, v, SCALE, bool(causal))
        got = dt_bwd(cuda, do, o, m, l, q, k, v, bool(causal))
        check(got, [z[f"{name}__{n}"] for n in ("dq", "dk", "dv")], name)


def test_flash_bwd_host_api_matches_device_api(cuda):
    import dirktensor_b200 as dt

    q, k, v = qkv(77, 1, 200, 2)
    do = randn(78, q.shape)
    o, m, l = oracle.flash_fwd(q, k, v, SCALE, True)
    gh = dt.flash_attention_backward(do, o, m, l, q, k, v, SCALE, True)
    gd = dt_bwd(cuda, do, o, m, l, q, k, v)
    for a, b in zip(gh, gd):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("B,T", [(1, 2048), (1, 4096), (2, 3000)])
def test_flash_bwd_full_size_vs_torch_autograd(cuda, B, T):
    """Config-1 sizes: torch fp32 autograd of softmax(scale QK^T + mask) V on the GPU."""
    import torch

    import dirktensor_b200 as dt

    H = 16
    g = torch.Generator(device=cuda)
    g.manual_seed(T + B)
    q, k, v, do = (torch.randn((B, T, H, 128), generator=g, device=cuda) for _ in range(4))
    fwd = dt.flash_attention_forward(q, k, v, SCALE, True)
    grads = dt.flash_attention_backward(do, fwd.output, fwd.softmax_m, fwd.softmax_l, q, k, v, SCALE, True)
    dt.check_device_error()
    qt, kt, vt = (t.detach().permute(0, 2, 1, 3).contiguous().requires_grad_(True) for t in (q, k, v))
    s = (qt @ kt.transpose(-1, -2)) * SCALE
    s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool, device=cuda), 1), float("-inf"))
    ot = torch.softmax(s, -1) @ vt
    ot.backward(do.permute(0, 2, 1, 3))
    for got, ref in zip(grads, (qt.grad, kt.grad, vt.grad)):
        ref = ref.permute(0, 2, 1, 3)
        err = float((got - ref).norm() / ref.norm())
        assert err < TOL_BWD_REL_L2, err
        assert bool(torch.isfinite(got).all())
