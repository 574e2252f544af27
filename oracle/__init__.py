"""TEST INFRASTRUCTURE (oracle) -- not part of the product.

ctypes bindings for
  * ``liboracle.so``: the C restatement of DirkTensor's attention hot path
    (``oracle.c``; every function there cites the reference file:line it follows);
  * ``_ref/libref_flash_<arch>.so``: the reference's own ``flash_attention_forward``
    and ``flash_attention_backward`` (FlashAttention.cpp:24-359) compiled in place
    against ``oracle/shims``.

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


def reference_dir() -> str:
    """The reference source tree: $DT_REFERENCE_DIR, else the Makefile's REF default."""
    env = os.environ.get("DT_REFERENCE_DIR")
    if env:
        return env
    r = subprocess.run(["make", "-s", "-C", HERE, "print-ref"], capture_output=True, text=True)
    return r.stdout.strip()


def reference_present() -> bool:
    d = reference_dir()
    return bool(d) and os.path.exists(os.path.join(d, "FlashAttention.cpp"))


def build(with_reference: bool | None = None) -> None:
    """Build liboracle.so, and the reference library when its sources exist."""
    targets = ["oracle"]
    if with_reference is None:
        with_reference = reference_present()
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
        L.or_sgemm.argtypes = [ctypes.c_int] * 5 + [ctypes.c_float, _f32p, ctypes.c_int, _f32p, ctypes.c_int,
                                                     ctypes.c_float, _f32p, ctypes.c_int]
        L.or_rmsnorm_rms.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_long, ctypes.c_int, ctypes.c_float]
        L.or_rmsnorm_bwd.argtypes = [_f32p] * 6 + [ctypes.c_long, ctypes.c_int]
        L.or_rope_bwd.argtypes = [_f32p, _f32p, ctypes.c_long, ctypes.c_long, ctypes.c_int, ctypes.c_int, _f32p,
                                  _f32p]
        L.or_flash_bwd.argtypes = [_f32p] * 10 + [ctypes.c_long, ctypes.c_long, ctypes.c_int, ctypes.c_int,
                                                  ctypes.c_float, ctypes.c_int]
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
        L.ref_flash_backward.restype = ctypes.c_double
        L.ref_flash_backward.argtypes = [_f32p] * 10 + [ctypes.c_long] * 4 + [ctypes.c_float, ctypes.c_int]
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


# ---------------------------------------------------------------------------
# Training path (backward): restatements of FlashAttention.cpp:185-359,
# OlmoAttention.cpp:149-330 and RMSNorm.cpp:24-41.
# ---------------------------------------------------------------------------

def sgemm(a, b, trans_a: bool, trans_b: bool, alpha: float = 1.0, c=None, beta: float = 0.0):
    """Row-major CBLAS sgemm: C = alpha * op(A) op(B) + beta * C."""
    a, b = _c(a), _c(b)
    M = a.shape[1] if trans_a else a.shape[0]
    K = a.shape[0] if trans_a else a.shape[1]
    N = b.shape[0] if trans_b else b.shape[1]
    if c is None:
        c = np.zeros((M, N), np.float32)
    lib().or_sgemm(int(trans_a), int(trans_b), M, N, K, alpha, a, a.shape[1], b, b.shape[1], beta, c, N)
    return c


def rmsnorm_rms(x, g, eps: float = 1e-6):
    """RMSNorm forward returning (y, rms per row)."""
    x = _c(x)
    rows = x.size // x.shape[-1]
    y = np.empty_like(x)
    rms = np.empty(rows, np.float32)
    lib().or_rmsnorm_rms(x, _c(g), y, rms, rows, x.shape[-1], eps)
    return y, rms


def rmsnorm_bwd(dy, y, g, rms, dg=None):
    """RMSNorm.cpp:24-36.  Returns (dx, dg) with dg accumulated into the given array."""
    dy, y = _c(dy), _c(y)
    dim = y.shape[-1]
    dx = np.empty_like(dy)
    if dg is None:
        dg = np.zeros(dim, np.float32)
    lib().or_rmsnorm_bwd(dy, y, _c(g), _c(rms), dx, dg, dy.size // dim, dim)
    return dx, dg


def rope_bwd(dy, sin_t=None, cos_t=None):
    """OlmoAttention.cpp:149-187.  dy: [B,T,H,D]."""
    dy = _c(dy)
    B, T, H, D = dy.shape
    if sin_t is None:
        sin_t, cos_t = rope_tables(T, D)
    dx = np.empty_like(dy)
    lib().or_rope_bwd(dy, dx, B, T, H, D, _c(sin_t), _c(cos_t))
    return dx


def flash_bwd(dout, out, m, l, q, k, v, scale: float, causal: bool = True):
    """Restated FlashAttention.cpp:185-359.  Returns (dq, dk, dv)."""
    args = [_c(a) for a in (dout, out, m, l, q, k, v)]
    B, T, H, D = args[4].shape
    dq, dk, dv = (np.empty_like(args[4]) for _ in range(3))
    lib().or_flash_bwd(*args, dq, dk, dv, B, T, H, D, scale, int(causal))
    return dq, dk, dv


def ref_flash_bwd(dout, out, m, l, q, k, v, scale: float, causal: bool = True, threads: int = 0):
    """The reference's own flash_attention_backward.  Returns (dq, dk, dv, seconds)."""
    L = ref_lib()
    if L is None:
        raise RuntimeError("reference flash library not built (oracle/_ref)")
    args = [_c(a) for a in (dout, out, m, l, q, k, v)]
    B, T, H, D = args[4].shape
    dq, dk, dv = (np.empty_like(args[4]) for _ in range(3))
    L.ref_set_threads(int(threads))
    secs = L.ref_flash_backward(*args, dq, dk, dv, B, T, H, D, scale, int(causal))
    if secs < 0:
        raise RuntimeError("reference flash_attention_backward raised")
    return dq, dk, dv, secs


def attention_layer_train(x, wq, wk, wv, wo, qg, kg, eps: float = 1e-6, theta: float = 500000.0,
                          n_heads: int = 16):
    """OlmoAttention::forward (OlmoAttention.cpp:56-108) keeping the activations
    its backward reads (OlmoAttention.h:28-38).  Returns (y, saved)."""
    x = _c(x)
    B, T, d = x.shape
    hd = d // n_heads
    x2 = x.reshape(-1, d)
    qp, kp, vp = linear(x2, wq), linear(x2, wk), linear(x2, wv)
    qn, rq = rmsnorm_rms(qp, qg, eps)
    kn, rk = rmsnorm_rms(kp, kg, eps)
    s_t, c_t = rope_tables(T, hd, theta)
    qr = rope(qn.reshape(B, T, n_heads, hd), s_t, c_t)
    kr = rope(kn.reshape(B, T, n_heads, hd), s_t, c_t)
    v4 = vp.reshape(B, T, n_heads, hd)
    scale = 1.0 / np.sqrt(np.float32(hd))
    o, m, l = flash_fwd(qr, kr, v4, float(scale), True)
    y = linear(o.reshape(-1, d), wo).reshape(B, T, d)
    saved = dict(x2=x2, qn=qn, kn=kn, rq=rq, rk=rk, qr=qr, kr=kr, v=v4, o=o, m=m, l=l, sin=s_t, cos=c_t,
                 scale=float(scale))
    return y, saved


def attention_layer_backward(dy, saved, wq, wk, wv, wo, qg, kg, n_heads: int = 16):
    """OlmoAttention::backward (OlmoAttention.cpp:189-312).  Returns (dx, grads)
    with grads = dict(q_proj, k_proj, v_proj, o_proj, q_norm, k_norm)."""
    dy = _c(dy)
    B, T, d = dy.shape
    hd = d // n_heads
    dy2 = dy.reshape(-1, d)
    a2 = saved["o"].reshape(-1, d)
    g = {}
    g["o_proj"] = sgemm(dy2, a2, True, False)                       # :201-205
    da = sgemm(dy2, wo, False, False).reshape(B, T, n_heads, hd)  # :207
    dq_r, dk_r, dv = flash_bwd(da, saved["o"], saved["m"], saved["l"], saved["qr"], saved["kr"], saved["v"],
                               saved["scale"], True)                # :219-221
    dq_n = rope_bwd(dq_r, saved["sin"], saved["cos"]).reshape(-1, d)  # :228-229
    dk_n = rope_bwd(dk_r, saved["sin"], saved["cos"]).reshape(-1, d)
    dqp, g["q_norm"] = rmsnorm_bwd(dq_n, saved["qn"], qg, saved["rq"])  # :236-237
    dkp, g["k_norm"] = rmsnorm_bwd(dk_n, saved["kn"], kg, saved["rk"])
    dv2 = dv.reshape(-1, d)
    x2 = saved["x2"]
    g["q_proj"] = sgemm(dqp, x2, True, False)                         # :250-254
    g["k_proj"] = sgemm(dkp, x2, True, False)
    g["v_proj"] = sgemm(dv2, x2, True, False)
    dx = sgemm(dqp, wq, False, False)                                  # :278-298
    sgemm(dkp, wk, False, False, c=dx, beta=1.0)
    sgemm(dv2, wv, False, False, c=dx, beta=1.0)
    return dx.reshape(B, T, d), g
