"""GPU: the attention kernel's fp32-Q path (dt_flash_fwd_qf32, used by dt_flash_fwd and
the head-parallel step) rounds the rows of Q to bf16 inside the kernel.  Both that
rounding and dt_cast_f32_bf16 are round-to-nearest-even, so every output must be
bit-identical to casting Q first and calling dt_flash_fwd_bf16 on the same K, V."""
import numpy as np
import pytest

from common import SCALE, qkv

pytestmark = pytest.mark.gpu


def _both(cuda, q, k, v, causal, out_bf16=False, row_pad=0, seq_lens=None):
    import torch

    import dirktensor_b200 as dt

    Q, K, V = (torch.from_numpy(a).to(cuda) for a in (q, k, v))
    Kb, Vb = dt.cast_bf16(K), dt.cast_bf16(V)
    B, T, H, D = Q.shape
    stride = H * D + row_pad
    sl = None if seq_lens is None else torch.tensor(seq_lens, dtype=torch.int32, device=cuda)
    res = []
    for qf in (True, False):
        out = torch.full((B, T, stride), 7.0, dtype=torch.bfloat16 if out_bf16 else torch.float32, device=cuda)
        m = torch.full((B, T, H), 3.0, device=cuda)
        l = torch.full((B, T, H), 5.0, device=cuda)
        if qf:
            dt.flash_attention_forward_qf32(Q, Kb, Vb, SCALE, causal, out=out, out_bf16=out_bf16,
                                            out_row_stride=stride, softmax_m=m, softmax_l=l, seq_lens=sl)
        else:
            dt.flash_attention_forward_bf16(dt.cast_bf16(Q), Kb, Vb, SCALE, causal, out=out, out_bf16=out_bf16,
                                            out_row_stride=stride, softmax_m=m, softmax_l=l, seq_lens=sl)
        dt.check_device_error()
        res.append([t.float().cpu().numpy() for t in (out, m, l)])
    return res


@pytest.mark.parametrize("B,T,H,causal", [(1, 1, 2, True), (1, 129, 2, True), (2, 300, 3, True),
                                          (1, 513, 1, False), (2, 1000, 2, True), (1, 2048, 4, True)])
def test_qf32_bit_identical_to_cast_then_bf16(cuda, B, T, H, causal):
    q, k, v = qkv(7000 + T + B, B, T, H)
    got, ref = _both(cuda, q, k, v, causal)
    for g, r, name in zip(got, ref, ("out", "m", "l")):
        assert np.array_equal(g, r), (name, float(np.max(np.abs(g - r))))


def test_qf32_bf16_output_row_stride_and_varlen(cuda):
    B, T, H = 3, 700, 2
    q, k, v = qkv(7100, B, T, H)
    got, ref = _both(cuda, q, k, v, True, out_bf16=True, row_pad=24, seq_lens=[700, 333, 1])
    for g, r, name in zip(got, ref, ("out", "m", "l")):
        assert np.array_equal(g, r), (name, float(np.max(np.abs(g - r))))
    # the padding columns of each output row are untouched
    assert np.all(got[0][:, :, H * 128:] == 7.0)
