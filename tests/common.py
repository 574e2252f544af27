"""Shared helpers for the test-suite: seeded inputs, error metrics, tolerances."""
from __future__ import annotations

import numpy as np

SCALE = 1.0 / np.sqrt(128.0)

# Tolerances of the bf16-operand / fp32-accumulate path against the fp32 CPU
# reference (calibrated against the fp64 truth; the fp32 reference itself sits
# at ~1e-6 of the truth).
TOL_ATTN_REL_L2 = 1e-2    # attention output, relative L2
TOL_ATTN_MAX_ABS = 5e-2   # attention output, max |diff|
TOL_M_ABS = 5e-2          # softmax_m (scaled-score units)
TOL_L_REL = 2e-2          # softmax_l, relative
TOL_LAYER_REL_L2 = 1.5e-2  # attention layer output y, relative L2
TOL_GEMM_REL_L2 = 1e-5    # GEMM vs fp32 matmul of the same bf16-rounded operands
TOL_BWD_REL_L2 = 2e-2    # attention gradients dQ, dK, dV, relative L2 (bf16 Q/K/V/dO/P/dS operands)
TOL_LAYER_BWD_REL_L2 = 3e-2  # layer backward: dx and the six weight gradients, relative L2


def randn(seed: int, shape, scale: float = 1.0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    a = rng.standard_normal(shape, dtype=np.float32)
    if scale != 1.0:
        a *= np.float32(scale)
    return a


def qkv(seed: int, B: int, T: int, H: int, D: int = 128):
    """Config-1/4 style inputs: Q, K, V ~ N(0,1) fp32 [B, T, H, D]."""
    return tuple(randn(seed * 3 + i, (B, T, H, D)) for i in range(3))


def layer_weights(seed: int, d: int = 2048):
    """Config-0 weights: projections N(0, 0.02), norm gains 1 + N(0, 0.02)."""
    ws = [randn(seed * 10 + i, (d, d), 0.02) for i in range(4)]
    gains = [1.0 + randn(seed * 10 + 4 + i, (d,), 0.02) for i in range(2)]
    return ws + [g.astype(np.float32) for g in gains]


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def max_abs(a, b) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)))) if np.size(a) else 0.0


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bf16, returned as float32."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def model_layer_weights(seed: int, d: int = 2048, hidden: int = 8192):
    """One OLMo-2 block's weights (config 3): projections N(0, 0.02), norm gains 1 + N(0, 0.02)."""
    shapes = {"q_proj": (d, d), "k_proj": (d, d), "v_proj": (d, d), "o_proj": (d, d), "gate_proj": (hidden, d),
              "up_proj": (hidden, d), "down_proj": (d, hidden)}
    w = {k: randn(seed * 31 + i, s, 0.02) for i, (k, s) in enumerate(shapes.items())}
    for i, k in enumerate(("q_norm", "k_norm", "post_attention_norm", "post_feedforward_norm")):
        w[k] = (1 + randn(seed * 31 + 20 + i, (d,), 0.02)).astype(np.float32)
    return w


def model_weights(seed: int, n_layers: int, vocab: int, distinct: int = 2):
    """Embedding, blocks, final norm gain and LM head.  `distinct` weight sets are
    generated and repeated over the layers (generation time, not arithmetic,
    is what this saves)."""
    base = [model_layer_weights(seed + i) for i in range(min(distinct, n_layers))]
    layers = [base[i % len(base)] for i in range(n_layers)]
    embed = randn(seed + 100, (vocab, 2048), 0.02)
    lm_head = randn(seed + 101, (vocab, 2048), 0.02)
    final_norm = (1 + randn(seed + 102, (2048,), 0.02)).astype(np.float32)
    return embed, layers, final_norm, lm_head
