"""GPU parity of the tcgen05 flash-attention kernel through the C ABI.

Compares against the oracle (C restatement of FlashAttention.cpp:24-182), the
golden vectors of the reference's own build, and, at the configuration sizes
(T up to 6144, B=16), an fp64 truth on sampled rows plus a causality property.
Tolerances (bf16 operands, fp32 accumulate/softmax) are in tests/common.py."""
import os

import numpy as np
import pytest

import oracle
from common import (SCALE, TOL_ATTN_MAX_ABS, TOL_ATTN_REL_L2, TOL_L_REL, TOL_M_ABS, qkv, rel_l2)

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "flash_ref.npz")


def dt_flash(cuda, q, k, v, causal=True):
    import torch

    import dirktensor_b200 as dt

    Q, K, V = (torch.from_numpy(a).to(cuda) for a in (q, k, v))
    r = dt.flash_attention_forward(Q, K, V, SCALE, causal)
    dt.check_device_error()
    return r.output.cpu().numpy(), r.softmax_m.cpu().numpy(), r.softmax_l.cpu().numpy()


def assert_close(o, m, l, ro, rm, rl):
    assert rel_l2(o, ro) < TOL_ATTN_REL_L2, rel_l2(o, ro)
    assert np.max(np.abs(o - ro)) < TOL_ATTN_MAX_ABS, np.max(np.abs(o - ro))
    assert np.max(np.abs(m - rm)) < TOL_M_ABS, np.max(np.abs(m - rm))
    assert np.max(np.abs(l - rl) / np.abs(rl)) < TOL_L_REL, np.max(np.abs(l - rl) / np.abs(rl))


@pytest.mark.parametrize("T", [1, 2, 63, 64, 65, 127, 128, 129, 255, 256, 257, 300, 383, 384, 511, 512, 513])
def test_flash_edge_lengths_vs_oracle(cuda, T):
    q, k, v = qkv(1000 + T, 1, T, 2)
    o, m, l = dt_flash(cuda, q, k, v)
    ro, rm, rl = oracle.flash_fwd(q, k, v, SCALE, True)
    assert_close(o, m, l, ro, rm, rl)


@pytest.mark.parametrize("B,T,H,causal", [(2, 700, 3, True), (1, 1024, 16, True), (1, 520, 2, False),
                                          (3, 129, 1, False), (1, 1000, 4, True)])
def test_flash_shapes_vs_oracle(cuda, B, T, H, causal):
    q, k, v = qkv(2000 + T + B, B, T, H)
    o, m, l = dt_flash(cuda, q, k, v, causal)
    ro, rm, rl = oracle.flash_fwd(q, k, v, SCALE, causal)
    assert_close(o, m, l, ro, rm, rl)


def test_flash_vs_reference_golden(cuda):
    z = np.load(GOLDEN)
    names = sorted({k.split("__")[0] for k in z.files})
    assert names
    for name in names:
        seed, B, T, H, causal = (int(x) for x in z[f"{name}__meta"])
        q, k, v = qkv(seed, B, T, H)
        o, m, l = dt_flash(cuda, q, k, v, bool(causal))
        assert_close(o, m, l, z[f"{name}__o"], z[f"{name}__m"], z[f"{name}__l"])


def test_flash_host_api_matches_device_api(cuda):
    import dirktensor_b200 as dt

    q, k, v = qkv(7, 2, 333, 4)
    o, m, l = dt_flash(cuda, q, k, v)
    ho, hm, hl = dt.flash_attention_forward(q, k, v, SCALE, True)
    assert np.array_equal(o, ho) and np.array_equal(m, hm) and np.array_equal(l, hl)


def test_flash_empty_inputs(cuda):
    import torch

    import dirktensor_b200 as dt

    for shape in [(0, 16, 2, 128), (1, 0, 2, 128), (1, 16, 0, 128)]:
        x = torch.zeros(shape, device=cuda)
        r = dt.flash_attention_forward(x, x, x, SCALE, True)
        assert r.output.shape == shape
    dt.check_device_error()


def _sample_rows(rng, B, T, H, n):
    rows = np.stack([rng.integers(0, B, n), rng.integers(0, T, n), rng.integers(0, H, n)], 1)
    rows[:8, 1] = [0, 1, 127, 128, 255, 256, T - 2, T - 1]  # tile edges and the last rows
    return rows


@pytest.mark.parametrize("B,T", [(1, 2048), (1, 4096), (1, 6144), (16, 6144)])
def test_flash_full_size_sampled_rows_vs_fp64(cuda, B, T):
    """Configuration sizes (config 1 sweep, config 4): sampled rows against fp64."""
    H = 16
    q, k, v = qkv(3000 + T + B, B, T, H)
    o, m, l = dt_flash(cuda, q, k, v)
    rows = _sample_rows(np.random.default_rng(T + B), B, T, H, 256)
    to, tm, tl = oracle.attention_rows_f64(q, k, v, rows, SCALE, True)
    go = o[rows[:, 0], rows[:, 1], rows[:, 2]]
    gm = m[rows[:, 0], rows[:, 1], rows[:, 2]]
    gl = l[rows[:, 0], rows[:, 1], rows[:, 2]]
    assert rel_l2(go, to) < TOL_ATTN_REL_L2
    assert np.max(np.abs(go - to)) < TOL_ATTN_MAX_ABS
    assert np.max(np.abs(gm - tm)) < TOL_M_ABS
    assert np.max(np.abs(gl - tl) / tl) < TOL_L_REL
    assert np.isfinite(o).all()


def test_flash_causality_property(cuda):
    """Changing keys/values after position t leaves rows <= t bit-identical."""
    B, T, H, t0 = 1, 2048, 16, 1000
    q, k, v = qkv(4242, B, T, H)
    o1, m1, l1 = dt_flash(cuda, q, k, v)
    k2, v2 = k.copy(), v.copy()
    k2[:, t0 + 1:] = np.random.default_rng(1).standard_normal(k2[:, t0 + 1:].shape, dtype=np.float32)
    v2[:, t0 + 1:] *= -3.0
    o2, m2, l2 = dt_flash(cuda, q, k2, v2)
    assert np.array_equal(o1[:, :t0 + 1], o2[:, :t0 + 1])
    assert np.array_equal(m1[:, :t0 + 1], m2[:, :t0 + 1])
    assert not np.array_equal(o1[:, t0 + 1:], o2[:, t0 + 1:])


def test_flash_linearity_in_v(cuda):
    """softmax(.)V is linear in V: O(V1 + V2) ~ O(V1) + O(V2) (bf16 rounding aside)."""
    q, k, v1 = qkv(77, 1, 1500, 4)
    v2 = qkv(78, 1, 1500, 4)[2]
    oa, _, _ = dt_flash(cuda, q, k, v1)
    ob, _, _ = dt_flash(cuda, q, k, v2)
    oc, _, _ = dt_flash(cuda, q, k, v1 + v2)
    assert rel_l2(oc, oa + ob) < TOL_ATTN_REL_L2
