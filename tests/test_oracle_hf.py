"""Independent pin of the oracle's layer and model restatements: HF transformers'
Olmo2Attention and Olmo2ForCausalLM (transformers 5.5, torch CPU fp32), built
from an Olmo2Config with the OLMo-2-0425-1B sizes -- no checkpoint, no network --
and given the same seeded weights as the oracle.

Olmo2Attention normalises q and k over all num_heads * head_dim = 2048 dims
before RoPE, as the reference does (OlmoAttention.cpp:70,76; RMSNorm.cpp:15-22),
and its decoder layer is the reference's post-norm block (OlmoBlock.cpp:13-21):
h = x + norm(attn(x)); out = h + norm(mlp(h)).

RoPE tables.  The reference computes sin/cos in double and casts to float
(OlmoAttention.cpp:18-36); HF computes them in float32.  The strict checks feed
HF the reference's double-derived tables (the oracle's `rope_tables`, itself
pinned to numpy double in test_oracle.py) through HF's own position_embeddings
argument, so that every other step -- projections, norm, rotate-half, masking,
softmax, O projection, MLP, residuals, final norm, LM head -- is HF's code.  A
second check runs HF's own fp32 tables and bounds the difference they make.

Tolerances: <= 1e-5 relative L2 with the reference's tables (the two fp32
computations differ only in summation order); <= 1e-4 with HF's fp32 tables."""
import numpy as np
import pytest

import oracle
from common import layer_weights, model_weights, rel_l2

torch = pytest.importorskip("torch")
m2 = pytest.importorskip("transformers.models.olmo2.modeling_olmo2")
from transformers import Olmo2Config  # noqa: E402

TOL_STRICT = 1e-5
TOL_HF_TABLES = 1e-4


def config(n_layers=1, vocab=100352):
    return Olmo2Config(hidden_size=2048, num_attention_heads=16, num_key_value_heads=16, intermediate_size=8192,
                       num_hidden_layers=n_layers, vocab_size=vocab, rms_norm_eps=1e-6,
                       rope_parameters={"rope_type": "default", "rope_theta": 500000.0},
                       max_position_embeddings=8192, attention_bias=False, attention_dropout=0.0,
                       tie_word_embeddings=False, attn_implementation="eager")


def ref_position_embeddings(T, B=1):
    """The reference's RoPE tables (double -> float) in HF's (cos, sin) [B, T, 128] form."""
    s, c = oracle.rope_tables(T)
    cos = torch.from_numpy(c)[None].expand(B, T, 128).contiguous()
    sin = torch.from_numpy(s)[None].expand(B, T, 128).contiguous()
    return cos, sin


def causal_mask(T):
    return torch.full((T, T), float("-inf")).triu(1)[None, None]


def hf_attention(cfg, wq, wk, wv, wo, qg, kg):
    attn = m2.Olmo2Attention(cfg, layer_idx=0).eval()
    with torch.no_grad():
        for lin, w in ((attn.q_proj, wq), (attn.k_proj, wk), (attn.v_proj, wv), (attn.o_proj, wo)):
            lin.weight.copy_(torch.from_numpy(w))
        attn.q_norm.weight.copy_(torch.from_numpy(qg))
        attn.k_norm.weight.copy_(torch.from_numpy(kg))
    return attn


def test_attention_layer_matches_hf_olmo2attention():
    """Configuration 0: B=1, T=512, d_model 2048, 16 x 128, x ~ N(0, 1)."""
    torch.set_num_threads(max(1, torch.get_num_threads()))
    cfg = config()
    wq, wk, wv, wo, qg, kg = layer_weights(21)
    B, T = 1, 512
    x = np.random.default_rng(5).standard_normal((B, T, 2048), dtype=np.float32)
    attn = hf_attention(cfg, wq, wk, wv, wo, qg, kg)
    xt = torch.from_numpy(x)
    with torch.no_grad():
        y_hf, _ = attn(xt, ref_position_embeddings(T, B), causal_mask(T))
        rot = m2.Olmo2RotaryEmbedding(cfg)
        y_hf_tables, _ = attn(xt, rot(xt, torch.arange(T)[None].expand(B, T)), causal_mask(T))
    y_or = oracle.attention_layer(x, wq, wk, wv, wo, qg, kg)
    err = rel_l2(y_or, y_hf.numpy())
    assert err <= TOL_STRICT, err
    err_tables = rel_l2(y_or, y_hf_tables.numpy())
    assert err_tables <= TOL_HF_TABLES, err_tables


def test_attention_layer_matches_hf_batched_non_square():
    """B=2, T=300 (not a multiple of the oracle's 256-row blocks)."""
    cfg = config()
    wq, wk, wv, wo, qg, kg = layer_weights(22)
    B, T = 2, 300
    x = np.random.default_rng(6).standard_normal((B, T, 2048), dtype=np.float32)
    attn = hf_attention(cfg, wq, wk, wv, wo, qg, kg)
    with torch.no_grad():
        y_hf, _ = attn(torch.from_numpy(x), ref_position_embeddings(T, B), causal_mask(T))
    err = rel_l2(oracle.attention_layer(x, wq, wk, wv, wo, qg, kg), y_hf.numpy())
    assert err <= TOL_STRICT, err


def hf_model(n_layers, embed, layers, final_norm, lm_head):
    cfg = config(n_layers, embed.shape[0])
    with torch.device("meta"):
        model = m2.Olmo2ForCausalLM(cfg)
    model = model.to_empty(device="cpu").eval()
    names = {"q_proj": "self_attn.q_proj", "k_proj": "self_attn.k_proj", "v_proj": "self_attn.v_proj",
             "o_proj": "self_attn.o_proj", "q_norm": "self_attn.q_norm", "k_norm": "self_attn.k_norm",
             "post_attention_norm": "post_attention_layernorm", "gate_proj": "mlp.gate_proj",
             "up_proj": "mlp.up_proj", "down_proj": "mlp.down_proj",
             "post_feedforward_norm": "post_feedforward_layernorm"}
    sd = {"model.embed_tokens.weight": embed, "model.norm.weight": final_norm, "lm_head.weight": lm_head}
    for i, lw in enumerate(layers):
        for k, stem in names.items():
            sd[f"model.layers.{i}.{stem}.weight"] = lw[k]
    model.load_state_dict({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in sd.items()}, strict=False,
                          assign=True)
    # the non-persistent buffers (RoPE inverse frequencies) are not in the state dict: rebuild them
    model.model.rotary_emb = m2.Olmo2RotaryEmbedding(cfg)
    return model


def test_model_matches_hf_olmo2forcausallm():
    """Configuration-3 architecture: 16 layers, d_model 2048, SwiGLU 8192, vocab
    100352, on B=2 sequences of T=96 token ids uniform in [0, 100278)."""
    n_layers, vocab, B, T = 16, 100352, 2, 96
    embed, layers, final_norm, lm_head = model_weights(41, n_layers, vocab, distinct=4)
    ids = np.random.default_rng(41).integers(0, 100278, (B, T)).astype(np.uint32)
    model = hf_model(n_layers, embed, layers, final_norm, lm_head)
    cos, sin = ref_position_embeddings(T, B)
    # every layer reads the reference's double-derived tables
    model.model.rotary_emb.forward = lambda x, position_ids: (cos, sin)
    with torch.no_grad():
        out = model(input_ids=torch.from_numpy(ids.astype(np.int64)), attention_mask=None, use_cache=False)
    got = out.logits.float().numpy()
    ref = oracle.model_forward(ids, embed, layers, final_norm, lm_head)
    err = rel_l2(ref, got)
    assert err <= TOL_STRICT, err
    assert float(np.mean(ref.argmax(-1) == got.argmax(-1))) == 1.0
