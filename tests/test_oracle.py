"""CPU tests: the oracle (C restatement) pinned to the reference.

Pins: golden vectors produced by the reference's own flash_attention_forward
(tests/golden/flash_ref.npz), the reference library itself when it was built
here (oracle/_ref), and an fp64 truth."""
import os

import numpy as np
import pytest

import oracle
from common import SCALE, qkv, randn, rel_l2

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "flash_ref.npz")


def golden_cases():
    z = np.load(GOLDEN)
    names = sorted({k.split("__")[0] for k in z.files})
    return z, names


def _checksum(*arrs):
    return float(sum(np.sum(a.astype(np.float64) * (1 + np.arange(a.size).reshape(a.shape) % 7)) for a in arrs))


@pytest.mark.parametrize("name", golden_cases()[1])
def test_oracle_matches_reference_golden(name):
    z = np.load(GOLDEN)
    seed, B, T, H, causal = (int(x) for x in z[f"{name}__meta"])
    q, k, v = qkv(seed, B, T, H)
    assert _checksum(q, k, v) == pytest.approx(float(z[f"{name}__checksum"][0]), rel=1e-12), "input generator drifted"
    o, m, l = oracle.flash_fwd(q, k, v, SCALE, bool(causal))
    assert np.max(np.abs(o - z[f"{name}__o"])) < 1e-5
    assert np.max(np.abs(m - z[f"{name}__m"])) < 1e-5
    assert np.max(np.abs(l - z[f"{name}__l"]) / np.abs(z[f"{name}__l"])) < 1e-5


@pytest.mark.parametrize("B,T,H,causal", [(1, 200, 2, True), (2, 333, 1, True), (1, 130, 2, False)])
def test_oracle_matches_fp64_truth(B, T, H, causal):
    q, k, v = qkv(99 + T, B, T, H)
    o, m, l = oracle.flash_fwd(q, k, v, SCALE, causal)
    rows = np.array([(b, t, h) for b in range(B) for t in range(T) for h in range(H)])
    to, tm, tl = oracle.attention_rows_f64(q, k, v, rows, SCALE, causal)
    assert np.max(np.abs(o.reshape(-1, 128) - to)) < 1e-5
    assert np.max(np.abs(m.reshape(-1) - tm)) < 1e-5
    assert np.max(np.abs(l.reshape(-1) - tl) / tl) < 1e-5


@pytest.mark.skipif(oracle.ref_lib() is None, reason="reference library not built (no reference sources)")
def test_oracle_matches_reference_library_live():
    q, k, v = qkv(5, 2, 600, 2)
    o, m, l = oracle.flash_fwd(q, k, v, SCALE, True)
    ro, rm, rl, _ = oracle.ref_flash_fwd(q, k, v, SCALE, True)
    assert np.max(np.abs(o - ro)) < 1e-5
    assert np.max(np.abs(m - rm)) < 1e-5
    assert np.max(np.abs(l - rl) / rl) < 1e-5


def test_rope_tables_against_numpy_double():
    s, c = oracle.rope_tables(300, 128, 500000.0)
    i = np.arange(64, dtype=np.float64)
    inv = 1.0 / np.power(500000.0, 2 * i / 128.0)
    ang = np.arange(300, dtype=np.float64)[:, None] * np.concatenate([inv, inv])[None, :]
    assert np.array_equal(s, np.sin(ang).astype(np.float32))
    assert np.array_equal(c, np.cos(ang).astype(np.float32))


def test_rmsnorm_and_rope_against_numpy():
    x = randn(1, (3, 7, 2048))
    g = (1 + randn(2, (2048,), 0.02)).astype(np.float32)
    y = oracle.rmsnorm(x, g)
    x64 = x.astype(np.float64)
    ref = x64 / np.sqrt((x64 ** 2).mean(-1, keepdims=True) + 1e-6) * g
    assert rel_l2(y, ref) < 1e-6
    xr = randn(3, (2, 9, 16, 128))
    s, c = oracle.rope_tables(9)
    yr = oracle.rope(xr, s, c)
    x1, x2 = xr[..., :64].astype(np.float64), xr[..., 64:].astype(np.float64)
    cs, sn = c[None, :, None, :], s[None, :, None, :]
    ref = np.concatenate([x1 * cs[..., :64] - x2 * sn[..., :64], x2 * cs[..., 64:] + x1 * sn[..., 64:]], -1)
    assert rel_l2(yr, ref) < 1e-6


def test_attention_layer_composes_stages():
    """The restated OlmoAttention::forward equals the stage-by-stage composition."""
    B, T = 1, 40
    x = randn(7, (B, T, 2048))
    wq, wk, wv, wo, qg, kg = (randn(20 + i, (2048, 2048), 0.02) for i in range(4)), None, None, None, None, None
    ws = [randn(20 + i, (2048, 2048), 0.02) for i in range(4)]
    qg = (1 + randn(30, (2048,), 0.02)).astype(np.float32)
    kg = (1 + randn(31, (2048,), 0.02)).astype(np.float32)
    y, inter = oracle.attention_layer(x, *ws, qg, kg, intermediates=True)
    s, c = oracle.rope_tables(T)
    q = oracle.rope(oracle.rmsnorm(oracle.linear(x, ws[0]), qg).reshape(B, T, 16, 128), s, c)
    k = oracle.rope(oracle.rmsnorm(oracle.linear(x, ws[1]), kg).reshape(B, T, 16, 128), s, c)
    v = oracle.linear(x, ws[2]).reshape(B, T, 16, 128)
    a, _, _ = oracle.flash_fwd(q, k, v, SCALE, True)
    ref = oracle.linear(a.reshape(B, T, 2048), ws[3])
    assert np.max(np.abs(y - ref)) < 1e-5
    assert np.max(np.abs(inter["q"].reshape(q.shape) - q)) < 1e-6
