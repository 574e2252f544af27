"""GPU parity of the projection GEMM, the norm/RoPE prologue and the whole
attention layer (OlmoAttention::forward, OlmoAttention.cpp:56-108) through the C ABI."""
import numpy as np
import pytest

import oracle
from common import (TOL_GEMM_REL_L2, TOL_LAYER_REL_L2, bf16_round, layer_weights, randn, rel_l2)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (200, 300, 136), (512, 6144, 2048), (1000, 2048, 2048),
                                   (1, 40, 8), (4096, 2304, 1024), (3000, 520, 8192), (200, 20000, 64)])
def test_gemm_vs_torch_fp32(cuda, M, N, K):
    import torch

    import dirktensor_b200 as dt

    a = torch.from_numpy(randn(M + N, (M, K))).to(cuda).to(torch.bfloat16)
    b = torch.from_numpy(randn(K + 1, (N, K), 0.05)).to(cuda).to(torch.bfloat16)
    c = dt.gemm_bf16_tn(a, b)
    # bf16 rows must stay 16-byte aligned: pad the leading dimension to a multiple of 8
    cb = dt.gemm_bf16_tn(a, b, out=torch.empty((M, (N + 7) // 8 * 8), dtype=torch.bfloat16, device=cuda),
                         out_bf16=True)[:, :N]
    dt.check_device_error()
    ref = a.float() @ b.float().t()
    assert rel_l2(c.cpu().numpy(), ref.cpu().numpy()) < TOL_GEMM_REL_L2
    assert rel_l2(cb.float().cpu().numpy(), ref.cpu().numpy()) < 5e-3


@pytest.mark.parametrize("a_mn,b_mn", [(0, 1), (1, 1), (1, 0)])
@pytest.mark.parametrize("M,N,K", [(2048, 2048, 1000), (6144, 2048, 520), (256, 384, 64), (136, 200, 300),
                                   (1000, 2048, 2048)])
def test_gemm_transposed_operands_vs_torch_fp32(cuda, a_mn, b_mn, M, N, K):
    """The training path's products: dW = dY^T X (both operands MN-major, added
    into the gradient) and dX = dY W (B MN-major)."""
    import torch

    import dirktensor_b200 as dt

    if (a_mn and M % 8) or (b_mn and N % 8) or ((not a_mn or not b_mn) and K % 8):
        pytest.skip("shape not supported by this operand layout")
    a = torch.from_numpy(randn(M + K, (M, K))).to(cuda).to(torch.bfloat16)
    b = torch.from_numpy(randn(N + K, (N, K), 0.05)).to(cuda).to(torch.bfloat16)
    a_in = a.t().contiguous() if a_mn else a
    b_in = b.t().contiguous() if b_mn else b
    ref = a.float() @ b.float().t()
    c = dt.gemm_bf16(a_in, b_in, a_mn=bool(a_mn), b_mn=bool(b_mn))
    base = torch.from_numpy(randn(7, (M, N))).to(cuda)
    acc = base.clone()
    dt.gemm_bf16(a_in, b_in, a_mn=bool(a_mn), b_mn=bool(b_mn), out=acc, accumulate=True)
    dt.check_device_error()
    assert rel_l2(c.cpu().numpy(), ref.cpu().numpy()) < TOL_GEMM_REL_L2
    assert rel_l2(acc.cpu().numpy(), (base + ref).cpu().numpy()) < TOL_GEMM_REL_L2


def test_cast_is_round_to_nearest_even(cuda):
    import torch

    import dirktensor_b200 as dt

    x = randn(5, (3, 1000, 4))
    y = dt.cast_bf16(torch.from_numpy(x).to(cuda))
    assert np.array_equal(y.float().cpu().numpy(), bf16_round(x))
    assert torch.equal(y, torch.from_numpy(x).to(cuda).to(torch.bfloat16))


def test_prologue_vs_oracle(cuda):
    import torch

    import dirktensor_b200 as dt

    B, T = 2, 300
    qkv = randn(11, (B * T, 3 * 2048))
    qg = (1 + randn(12, (2048,), 0.02)).astype(np.float32)
    kg = (1 + randn(13, (2048,), 0.02)).astype(np.float32)
    dq = torch.from_numpy(qkv).to(cuda)
    qo, ko, vo = dt.qk_norm_rope(dq[:, :2048], dq[:, 2048:4096], dq[:, 4096:], torch.from_numpy(qg).to(cuda),
                                 torch.from_numpy(kg).to(cuda), B, T)
    dt.check_device_error()
    s, c = oracle.rope_tables(T)
    rq = oracle.rope(oracle.rmsnorm(qkv[:, :2048], qg).reshape(B, T, 16, 128), s, c).reshape(B * T, 2048)
    rk = oracle.rope(oracle.rmsnorm(qkv[:, 2048:4096], kg).reshape(B, T, 16, 128), s, c).reshape(B * T, 2048)
    # bf16 outputs: within one bf16 rounding of the fp32 oracle
    for got, ref in ((qo, rq), (ko, rk), (vo, qkv[:, 4096:])):
        g = got.float().cpu().numpy()
        assert np.max(np.abs(g - ref) / (np.abs(ref) + 1e-3)) < 2 ** -8
        assert rel_l2(g, ref) < 3e-3


def _layer(cuda, seed, B, T, seq_lens=None):
    import torch

    import dirktensor_b200 as dt

    ws = layer_weights(seed)
    x = randn(seed + 1, (B, T, 2048))
    attn = dt.OlmoAttention.from_weights(*ws, device=cuda.index or 0)
    y = attn.forward(torch.from_numpy(x).to(cuda), seq_lens=seq_lens)
    dt.check_device_error()
    return ws, x, attn, y.cpu().numpy()


def test_layer_config0_vs_oracle(cuda):
    """Config 0: B=1, T=512 attention layer vs the restated OlmoAttention::forward."""
    ws, x, attn, y = _layer(cuda, 100, 1, 512)
    ref = oracle.attention_layer(x, *ws)
    assert rel_l2(y, ref) < TOL_LAYER_REL_L2, rel_l2(y, ref)
    assert np.isfinite(y).all()
    # host-buffer entry point gives the same result
    yh = attn.forward(x)
    assert np.array_equal(yh, y)


def test_layer_small_batches_vs_oracle(cuda):
    for B, T in [(2, 37), (1, 1), (3, 260)]:
        ws, x, attn, y = _layer(cuda, 200 + T, B, T)
        ref = oracle.attention_layer(x, *ws)
        assert rel_l2(y, ref) < TOL_LAYER_REL_L2, (B, T, rel_l2(y, ref))


@pytest.mark.parametrize("full", [False, True])
def test_layer_varlen_config2_vs_oracle(cuda, full):
    """Config 2: right-padded batch.  Valid rows match the reference run on each
    sequence alone; rows past a sequence's length are zeros."""
    if full:
        B, T = 8, 2048
        lens = np.random.default_rng(2).integers(256, 2049, B).astype(np.int32)
    else:
        B, T = 3, 300
        lens = np.array([300, 77, 129], np.int32)
    ws, x, attn, y = _layer(cuda, 300, B, T, seq_lens=lens)
    check = range(B) if not full else range(0, B, 3)
    for b in check:
        L = int(lens[b])
        ref = oracle.attention_layer(x[b:b + 1, :L], *ws)
        assert rel_l2(y[b:b + 1, :L], ref) < TOL_LAYER_REL_L2, (b, L, rel_l2(y[b:b + 1, :L], ref))
        assert np.all(y[b, L:] == 0)


def test_layer_from_npy_checkpoint(cuda, tmp_path):
    import torch

    import dirktensor_b200 as dt

    ws = layer_weights(400)
    names = ["q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm"]
    for n, w in zip(names, ws):
        np.save(tmp_path / f"model.layers.3.self_attn.{n}.weight.npy", w)
    attn = dt.OlmoAttention(str(tmp_path), 3, device=0)
    x = randn(401, (1, 64, 2048))
    y = attn.forward(torch.from_numpy(x).to(cuda)).cpu().numpy()
    y2 = dt.OlmoAttention.from_weights(*ws).forward(torch.from_numpy(x).to(cuda)).cpu().numpy()
    assert np.array_equal(y, y2)
    with pytest.raises(dt.DTError):
        dt.OlmoAttention(str(tmp_path), 4, device=0)
