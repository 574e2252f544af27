"""GPU parity of the full OLMo-2 prefill (configuration 3 architecture):
OlmoModel::forward (OlmoModel.cpp:25-48) with OlmoBlock (OlmoBlock.cpp:13-21),
OlmoMlp (OlmoMlp.cpp:26-63) and OlmoLmHead (OlmoLmHead.cpp:11-28), against the
oracle's restatement.  Weights N(0, 0.02), norm gains 1 + N(0, 0.02)."""
import numpy as np
import pytest

import oracle
from common import model_weights, rel_l2

pytestmark = pytest.mark.gpu

TOL_LOGITS_REL_L2 = 3e-2
KEYS = oracle.LAYER_KEYS


def compare(cuda, n_layers, vocab, B, T, seed):
    import torch

    import dirktensor_b200 as dt

    embed, layers, final_norm, lm_head = model_weights(seed, n_layers, vocab)
    ids = np.random.default_rng(seed).integers(0, min(vocab, 100278), (B, T)).astype(np.uint32)
    m = dt.OlmoModel.from_weights(embed, layers, final_norm, lm_head)
    got = m.forward(torch.from_numpy(ids.astype(np.int32)).to(cuda)).cpu().numpy()
    dt.check_device_error()
    ref = oracle.model_forward(ids, embed, layers, final_norm, lm_head)
    err = rel_l2(got, ref)
    top1 = float(np.mean(got.argmax(-1) == ref.argmax(-1)))
    return m, ids, got, ref, err, top1


def test_model_reduced_vs_oracle(cuda):
    m, ids, got, ref, err, top1 = compare(cuda, n_layers=2, vocab=1024, B=2, T=160, seed=7)
    assert err < TOL_LOGITS_REL_L2, err
    assert top1 > 0.9, top1
    # host-buffer entry point: same logits
    assert np.array_equal(m.forward(ids), got)


def test_model_full_architecture_16_layers(cuda):
    """Config-3 architecture (16 layers, vocab 100352) on a short batch."""
    m, ids, got, ref, err, top1 = compare(cuda, n_layers=16, vocab=100352, B=1, T=64, seed=11)
    assert err < TOL_LOGITS_REL_L2, err
    assert top1 > 0.8, top1
    assert np.isfinite(got).all()


def test_model_rejects_out_of_range_tokens(cuda):
    import dirktensor_b200 as dt

    embed, layers, final_norm, lm_head = model_weights(3, 1, 512)
    m = dt.OlmoModel.from_weights(embed, layers, final_norm, lm_head)
    with pytest.raises(dt.DTError, match="vocabulary"):
        m.forward(np.array([[1, 2, 600]], np.uint32))


def test_model_from_npy_checkpoint(cuda, tmp_path):
    import dirktensor_b200 as dt

    embed, layers, final_norm, lm_head = model_weights(5, 2, 256)
    np.save(tmp_path / "model.embed_tokens.weight.npy", embed)
    np.save(tmp_path / "model.norm.weight.npy", final_norm)
    np.save(tmp_path / "lm_head.weight.npy", lm_head)
    names = {"post_attention_norm": "post_attention_layernorm", "post_feedforward_norm": "post_feedforward_layernorm",
             "gate_proj": "mlp.gate_proj", "up_proj": "mlp.up_proj", "down_proj": "mlp.down_proj"}
    for i, lw in enumerate(layers):
        for k in KEYS:
            stem = names.get(k, "self_attn." + k)
            np.save(tmp_path / f"model.layers.{i}.{stem}.weight.npy", lw[k])
    m = dt.OlmoModel(str(tmp_path), n_layers=2)
    assert m.vocab == 256 and m.n_layers == 2 and m.hidden == 8192
    ids = np.random.default_rng(0).integers(0, 256, (1, 40)).astype(np.uint32)
    a = m.forward(ids)
    b = dt.OlmoModel.from_weights(embed, layers, final_norm, lm_head).forward(ids)
    assert np.array_equal(a, b)
