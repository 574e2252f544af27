"""TEST INFRASTRUCTURE (oracle) -- not part of the product.

ctypes bindings for
  * ``liboracle.so``: the C restatement of DirkTensor's attention hot path
    (``oracle.c``; every function there cites the reference file:line it follows);
  * ``_ref/libref_flash_<arch>.so``: the reference's own ``flash_attention_forward``
    (FlashAttention.cpp:24-182) compiled in place against ``oracle/shims``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs
may import this module.  The product (``dirktensor_b200``) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")

_lib = None
_ref = None


def build(with_reference: bool | None = None) -> None:
    """Build liboracle.so, and the reference library when its sources exist."""
    targets = ["oracle"]
    if with_reference is None:
        with_reference = os.path.exists("/root/reference/FlashAttention.cpp")
    if with_reference:
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE] + targets, check=True)


def _cpu_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return " avx512f " in (line.rstrip() + " ")
    except OSError:
        pass
    return False


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build(with_reference=False)
        L = ctypes.CDLL(path)
        L.or_set_threads.argtypes = [ctypes.c_int]
        L.or_rope_tables.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_double, _f32p, _f32p]
        L.or_rmsnorm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_long, ctypes.c_int, ctypes.c_float]
        L.or_rope.argtypes = [_f32p, _f32p, ctypes.c_long, ctypes.c_long, ctypes.c_int, ctypes.c_int, _f32p, _f32p]
        L.or_linear.argtypes = [_f32p, _f32p, _f32p, ctypes.c_long, ctypes.c_int, ctypes.c_int]
        L.or_flash_fwd.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_void_p, ctypes.c_void_p,
                                   ctypes.c_long, ctypes.c_long, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_float, ctypes.c_int]
        L.or_attention_rows_f64.argtypes = [_f32p, _f32p, _f32p, ctypes.c_long, ctypes.c_long, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_double, ctypes.c_int, _i64p, ctypes.c_long,
                                            _f64p, _f64p, _f64p]
        L.or_attention_layer.argtypes = [_f32p] * 8 + [ctypes.c_long, ctypes.c_long, ctypes.c_int, ctypes.c_int,
                                                       ctypes.c_float, ctypes.c_double] + [ctypes.c_void_p] * 4
        L.or_mlp.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_long, ctypes.c_int, ctypes.c_int]
        L.or_model_forward.argtypes = [ctypes.c_void_p, ctypes.c_long, ctypes.c_long, _f32p, ctypes.c_void_p,
                                       ctypes.c_int, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_float, ctypes.c_double, _f32p]
        L.or_set_threads(0)
        _lib = L
    return _lib


def ref_lib():
    """The reference's own flash_attention_forward, or None if it was not built."""
    global _ref
    if _ref is None:
        arch = "x86-64-v4" if _cpu_has_avx512() else "x86-64-v3"
        path = os.path.join(REF_DIR, f"libref_flash_{arch}.so")
        if not os.path.exists(path):
            return None
        L = ctypes.CDLL(path)
        L.ref_set_threads.argtypes = [ctypes.c_int]
        L.ref_get_threads.restype = ctypes.c_int
        L.ref_flash_forward.restype = ctypes.c_double
        L.ref_flash_forward.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_long, ctypes.c_long,
                                        ctypes.c_long, ctypes.c_long, ctypes.c_float, ctypes.c_int]
        L.arch = arch
        _ref = L
    return _ref


def _c(a, dt=np.float32):
    return np.ascontiguousarray(a, dtype=dt)


def set_threads(n: int) -> None:
    lib().or_set_threads(int(n))


def rope_tables(max_seq: int, head_dim: int = 128, theta: float = 500000.0):
    s = np.empty((max_seq, head_dim), np.float32)
    c = np.empty((max_seq, head_dim), np.float32)
    lib().or_rope_tables(max_seq, head_dim, theta, s, c)
    return s, c


def rmsnorm(x, g, eps: float = 1e-6):
    x = _c(x)
    y = np.empty_like(x)
    lib().or_rmsnorm(x, _c(g), y, x.size // x.shape[-1], x.shape[-1], eps)
    return y


def rope(x, sin_t=None, cos_t=None):
    """x: [B,T,H,D]."""
    x = _c(x)
    B, T, H, D = x.shape
    if sin_t is None:
        sin_t, cos_t = rope_tables(T, D)
    y = np.empty_like(x)
    lib().or_rope(x, y, B, T, H, D, _c(sin_t), _c(cos_t))
    return y


def linear(x, w):
    """y = x . w^T with x [M,K], w [N,K]."""
    x = _c(x)
    w = _c(w)
    M = x.size // x.shape[-1]
    y = np.empty(x.shape[:-1] + (w.shape[0],), np.float32)
    lib().or_linear(x, w, y, M, w.shape[0], w.shape[1])
    return y


def flash_fwd(q, k, v, scale: float, causal: bool = True):
    """Restated FlashAttention.cpp:24-182.  Returns (o, m, l)."""
    q, k, v = _c(q), _c(k), _c(v)
    B, T, H, D = q.shape
    o = np.empty_like(q)
    m = np.empty((B, T, H), np.float32)
    l = np.empty((B, T, H), np.float32)
    lib().or_flash_fwd(q, k, v, o, m.ctypes.data, l.ctypes.data, B, T, H, D, scale, int(causal))
    return o, m, l


def attention_rows_f64(q, k, v, rows, scale: float, causal: bool = True):
    """fp64 truth for the given (b, t, h) rows.  Returns (o [n,D], m [n], l [n])."""
    q, k, v = _c(q), _c(k), _c(v)
    B, T, H, D = q.shape
    rows = _c(np.asarray(rows).reshape(-1, 3), np.int64)
    n = rows.shape[0]
    o = np.empty((n, D), np.float64)
    m = np.empty(n, np.float64)
    l = np.empty(n, np.float64)
    lib().or_attention_rows_f64(q, k, v, B, T, H, D, scale, int(causal), rows, n, o, m, l)
    return o, m, l


def attention_layer(x, wq, wk, wv, wo, qg, kg, eps: float = 1e-6, theta: float = 500000.0,
                    n_heads: int = 16, intermediates: bool = False):
    """Restated OlmoAttention::forward (OlmoAttention.cpp:56-108).  x: [B,T,d]."""
    x = _c(x)
    B, T, d = x.shape
    y = np.empty_like(x)
    inter = [np.empty_like(x) for _ in range(4)] if intermediates else None
    ptrs = [a.ctypes.data for a in inter] if inter else [None] * 4
    lib().or_attention_layer(x, _c(wq), _c(wk), _c(wv), _c(wo), _c(qg), _c(kg), y, B, T, d, n_heads,
                             eps, theta, *ptrs)
    if intermediates:
        return y, dict(q=inter[0], k=inter[1], v=inter[2], a=inter[3])
    return y


def ref_flash_fwd(q, k, v, scale: float, causal: bool = True, threads: int = 0):
    """The reference's own flash_attention_forward.  Returns (o, m, l, seconds)."""
    L = ref_lib()
    if L is None:
        raise RuntimeError("reference flash library not built (oracle/_ref)")
    q, k, v = _c(q), _c(k), _c(v)
    B, T, H, D = q.shape
    o = np.empty_like(q)
    m = np.empty((B, T, H), np.float32)
    l = np.empty((B, T, H), np.float32)
    L.ref_set_threads(int(threads))
    secs = L.ref_flash_forward(q, k, v, o, m, l, B, T, H, D, scale, int(causal))
    if secs < 0:
        raise RuntimeError("reference flash_attention_forward raised")
    return o, m, l, secs


class _LayerW(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm", "post_attention_norm", "gate_proj", "up_proj",
        "down_proj", "post_feedforward_norm")]


LAYER_KEYS = ("q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm", "post_attention_norm", "gate_proj",
              "up_proj", "down_proj", "post_feedforward_norm")


def mlp(x, w_gate, w_up, w_down):
    """Restated OlmoMlp::forward (OlmoMlp.cpp:26-63).  x: [M, d]."""
    x = _c(x)
    M, d = x.shape
    hidden = w_up.shape[0]
    out = np.empty_like(x)
    lib().or_mlp(x, _c(w_gate), _c(w_up), _c(w_down), out, M, d, hidden)
    return out


def model_forward(ids, embed, layers, final_norm, lm_head, n_heads: int = 16, eps: float = 1e-6,
                  theta: float = 500000.0):
    """Restated OlmoModel::forward (OlmoModel.cpp:25-48).  ids: [B, T] uint32;
    layers: list of dicts with LAYER_KEYS.  Returns logits [B, T, vocab]."""
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    B, T = ids.shape
    embed = _c(embed)
    vocab, d = embed.shape
    hidden = layers[0]["up_proj"].shape[0]
    keep = []
    arr = (_LayerW * len(layers))()
    for i, lw in enumerate(layers):
        for k in LAYER_KEYS:
            a = _c(lw[k])
            keep.append(a)
            setattr(arr[i], k, a.ctypes.data)
    logits = np.empty((B, T, lm_head.shape[0]), np.float32)
    lib().or_model_forward(ids.ctypes.data, B, T, embed, ctypes.cast(arr, ctypes.c_void_p), len(layers),
                           _c(final_norm), _c(lm_head), lm_head.shape[0], d, n_heads, hidden, eps, theta, logits)
    return logits
