"""dirktensor_b200: B200-native (sm_100a) attention hot path of DirkTensor's OLMo-2-0425-1B.

QKV projection -> QK-RMSNorm -> RoPE -> causal flash attention -> O projection,
as hand-written tcgen05/TMA kernels behind the C ABI in include/dirktensor_b200.h.
"""
from ._lib import DTError, lib  # noqa: F401  (loads the CUDA library; raises if unbuilt)
from .attention import (  # noqa: F401
    FlashAttentionGradients,
    FlashAttentionResult,
    OlmoAttention,
    OlmoModel,
    cast_bf16,
    cast2_bf16,
    check_device_error,
    d_model,
    flash_attention_backward,
    flash_attention_forward,
    flash_attention_forward_bf16,
    flash_attention_forward_qf32,
    gemm_bf16,
    gemm_bf16_tn,
    head_dim,
    max_seq_len,
    n_heads,
    n_layers,
    qk_norm_rope,
    rms_eps,
    rope_tables,
    rope_theta,
)

lib()
