"""Host-side mirror of DirkTensor's attention interface over the C ABI.

``flash_attention_forward`` mirrors FlashAttention.h:15-21 (returns a
``FlashAttentionResult`` with ``output``, ``softmax_m``, ``softmax_l`` as in
FlashAttention.h:6-10) and ``OlmoAttention`` mirrors OlmoAttention.h:10-42
(constructed from a checkpoint folder and layer index, ``forward`` on
[B, T, d_model] activations).  Arguments may be CUDA torch tensors (device
path, runs on the current stream, no synchronisation) or numpy arrays (host
path: copies in, computes, copies out).  All compute runs in the CUDA library;
errors surface as ``DTError``.
"""
from __future__ import annotations

import ctypes
from typing import NamedTuple, Optional

import numpy as np

from ._lib import check, dt_attn_weights, dt_model_layer_weights, dt_model_weights, lib

# model_config.h:3-7
head_dim = 128
max_seq_len = 8192
d_model = 2048
n_heads = d_model // head_dim
n_layers = 16
rms_eps = 1e-6        # RMSNorm.h:10
rope_theta = 500000.0  # OlmoAttention.cpp:16


class FlashAttentionResult(NamedTuple):
    output: object     # [B, T, H, D]
    softmax_m: object  # [B, T, H] row max of the scaled scores
    softmax_l: object  # [B, T, H] sum of exp(s - m)


def _torch():
    import torch
    return torch


def _is_torch(x) -> bool:
    try:
        import torch
    except ImportError:
        return False
    return isinstance(x, torch.Tensor)


def _stream_ptr(device) -> int:
    torch = _torch()
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _need_cuda_f32(name, t, ndim):
    torch = _torch()
    if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous() and t.dim() == ndim):
        raise ValueError(f"{name} must be a contiguous float32 CUDA tensor with {ndim} dims")


_ws_cache: dict = {}


def _workspace(device, nbytes: int):
    torch = _torch()
    key = torch.device(device).index
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf


def flash_attention_forward(Q, K, V, scale: float, causal: bool = True) -> FlashAttentionResult:
    """Causal (or full) attention forward; drop-in for FlashAttention.h:15-21.

    Q, K, V: [B, T, H, D] float32, D = 128.  Operands are rounded to bf16 for
    the tensor cores; accumulation and softmax are fp32.
    """
    if _is_torch(Q):
        torch = _torch()
        for n, t in (("Q", Q), ("K", K), ("V", V)):
            _need_cuda_f32(n, t, 4)
        if not (Q.shape == K.shape == V.shape):
            raise ValueError("Q, K, V shapes differ")
        B, T, H, D = Q.shape
        out = torch.empty_like(Q)
        m = torch.empty((B, T, H), dtype=torch.float32, device=Q.device)
        l = torch.empty((B, T, H), dtype=torch.float32, device=Q.device)
        nbytes = lib().dt_flash_fwd_workspace_bytes(B, T, H, D)
        ws = _workspace(Q.device, nbytes)
        check(lib().dt_flash_fwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(), m.data_ptr(),
                                 l.data_ptr(), B, T, H, D, float(scale), int(bool(causal)), ws.data_ptr(),
                                 ws.numel(), _stream_ptr(Q.device)))
        return FlashAttentionResult(out, m, l)
    Q = np.ascontiguousarray(Q, dtype=np.float32)
    K = np.ascontiguousarray(K, dtype=np.float32)
    V = np.ascontiguousarray(V, dtype=np.float32)
    if Q.ndim != 4 or not (Q.shape == K.shape == V.shape):
        raise ValueError("Q, K, V must be [B, T, H, D] with equal shapes")
    B, T, H, D = Q.shape
    out = np.empty_like(Q)
    m = np.empty((B, T, H), np.float32)
    l = np.empty((B, T, H), np.float32)
    check(lib().dt_flash_fwd_host(Q.ctypes.data, K.ctypes.data, V.ctypes.data, out.ctypes.data, m.ctypes.data,
                                  l.ctypes.data, B, T, H, D, float(scale), int(bool(causal))))
    return FlashAttentionResult(out, m, l)


class FlashAttentionGradients(NamedTuple):
    """Mirror of FlashAttentionGradients (FlashAttention.h:27-31)."""
    d_Q: object
    d_K: object
    d_V: object


def flash_attention_backward(d_output, output, softmax_m, softmax_l, Q, K, V, scale: float,
                             causal: bool = True) -> FlashAttentionGradients:
    """Drop-in for flash_attention_backward (FlashAttention.h:33-43).

    All tensors float32: d_output, output, Q, K, V [B, T, H, D] (D = 128);
    softmax_m, softmax_l [B, T, H] as flash_attention_forward returns them.
    Operands are rounded to bf16 for the tensor cores; the softmax recomputation
    and D = rowsum(output * d_output) are fp32.
    """
    names = ("d_output", "output", "Q", "K", "V")
    if _is_torch(Q):
        torch = _torch()
        for n, t in zip(names, (d_output, output, Q, K, V)):
            _need_cuda_f32(n, t, 4)
        _need_cuda_f32("softmax_m", softmax_m, 3)
        _need_cuda_f32("softmax_l", softmax_l, 3)
        B, T, H, D = Q.shape
        for t in (d_output, output, K, V):
            if t.shape != Q.shape:
                raise ValueError("d_output, output, Q, K, V shapes differ")
        dq, dk, dv = (torch.empty_like(Q) for _ in range(3))
        nbytes = lib().dt_flash_bwd_workspace_bytes(B, T, H, D)
        ws = _workspace(Q.device, nbytes)
        check(lib().dt_flash_bwd(d_output.data_ptr(), output.data_ptr(), softmax_m.data_ptr(),
                                 softmax_l.data_ptr(), Q.data_ptr(), K.data_ptr(), V.data_ptr(), dq.data_ptr(),
                                 dk.data_ptr(), dv.data_ptr(), B, T, H, D, float(scale), int(bool(causal)),
                                 ws.data_ptr(), ws.numel(), _stream_ptr(Q.device)))
        return FlashAttentionGradients(dq, dk, dv)
    arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (d_output, output, softmax_m, softmax_l, Q, K, V)]
    B, T, H, D = arrs[4].shape
    for a in (arrs[0], arrs[1], arrs[5], arrs[6]):
        if a.shape != arrs[4].shape:
            raise ValueError("d_output, output, Q, K, V shapes differ")
    dq, dk, dv = (np.empty_like(arrs[4]) for _ in range(3))
    check(lib().dt_flash_bwd_host(*[a.ctypes.data for a in arrs], dq.ctypes.data, dk.ctypes.data, dv.ctypes.data,
                                  B, T, H, D, float(scale), int(bool(causal))))
    return FlashAttentionGradients(dq, dk, dv)


def flash_attention_forward_bf16(q, k, v, scale: float, causal: bool = True, out=None, out_bf16: bool = False,
                                 out_row_stride: Optional[int] = None, softmax_m=None, softmax_l=None,
                                 seq_lens=None):
    """Packed-operand form: q, k, v bf16 CUDA tensors [B, T, H, D]."""
    torch = _torch()
    for n, t in (("q", q), ("k", k), ("v", v)):
        if not (t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous() and t.dim() == 4):
            raise ValueError(f"{n} must be a contiguous bfloat16 CUDA tensor [B, T, H, D]")
    B, T, H, D = q.shape
    if out is None:
        out = torch.empty((B, T, H, D), dtype=torch.bfloat16 if out_bf16 else torch.float32, device=q.device)
        out_row_stride = H * D
    if out_row_stride is None:
        out_row_stride = H * D
    check(lib().dt_flash_fwd_bf16(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), int(out_bf16),
                                  int(out_row_stride), _ptr(softmax_m), _ptr(softmax_l), _ptr(seq_lens), B, T, H,
                                  D, float(scale), int(bool(causal)), _stream_ptr(q.device)))
    return out


def flash_attention_forward_qf32(q, k, v, scale: float, causal: bool = True, out=None, out_bf16: bool = False,
                                 out_row_stride: Optional[int] = None, softmax_m=None, softmax_l=None,
                                 seq_lens=None):
    """q float32, k and v bf16 CUDA tensors [B, T, H, D]: the attention kernel
    rounds the rows of q to bf16 itself (no separate cast pass over q)."""
    torch = _torch()
    if not (q.is_cuda and q.dtype == torch.float32 and q.is_contiguous() and q.dim() == 4):
        raise ValueError("q must be a contiguous float32 CUDA tensor [B, T, H, D]")
    for n, t in (("k", k), ("v", v)):
        if not (t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous() and t.shape == q.shape):
            raise ValueError(f"{n} must be a contiguous bfloat16 CUDA tensor shaped like q")
    B, T, H, D = q.shape
    if out is None:
        out = torch.empty((B, T, H, D), dtype=torch.bfloat16 if out_bf16 else torch.float32, device=q.device)
        out_row_stride = H * D
    if out_row_stride is None:
        out_row_stride = H * D
    check(lib().dt_flash_fwd_qf32(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), int(out_bf16),
                                  int(out_row_stride), _ptr(softmax_m), _ptr(softmax_l), _ptr(seq_lens), B, T, H,
                                  D, float(scale), int(bool(causal)), _stream_ptr(q.device)))
    return out


def cast_bf16(x):
    """bf16 copy of a float32 CUDA tensor (element count a multiple of 4)."""
    torch = _torch()
    _need_cuda_f32("x", x, x.dim())
    y = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    check(lib().dt_cast_f32_bf16(x.data_ptr(), y.data_ptr(), x.numel(), _stream_ptr(x.device)))
    return y


def cast2_bf16(x, y):
    """bf16 copies of two float32 CUDA tensors of one element count, in one launch."""
    torch = _torch()
    _need_cuda_f32("x", x, x.dim())
    _need_cuda_f32("y", y, y.dim())
    if x.numel() != y.numel():
        raise ValueError("x and y must have the same number of elements")
    xb = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    yb = torch.empty(y.shape, dtype=torch.bfloat16, device=y.device)
    check(lib().dt_cast2_f32_bf16(x.data_ptr(), y.data_ptr(), xb.data_ptr(), yb.data_ptr(), x.numel(),
                                  _stream_ptr(x.device)))
    return xb, yb


def gemm_bf16_tn(A, B, out_bf16: bool = False, out=None):
    """C = A . B^T with A [M, K], B [N, K] bf16 CUDA tensors."""
    torch = _torch()
    M, K = A.shape
    N = B.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16 if out_bf16 else torch.float32, device=A.device)
    check(lib().dt_gemm_bf16_tn(A.data_ptr(), B.data_ptr(), out.data_ptr(), int(out_bf16), M, N, K, out.stride(0),
                                _stream_ptr(A.device)))
    return out


def gemm_bf16(A, B, a_mn: bool = False, b_mn: bool = False, out=None, accumulate: bool = False,
              out_bf16: bool = False):
    """C (+)= op(A) . op(B)^T with bf16 CUDA operands.  A is [M, K] (a_mn False)
    or stored [K, M] (a_mn True); B is [N, K] (b_mn False) or stored [K, N]
    (b_mn True).  accumulate adds into the given fp32 `out`."""
    torch = _torch()
    M, K = (A.shape[1], A.shape[0]) if a_mn else (A.shape[0], A.shape[1])
    N = B.shape[1] if b_mn else B.shape[0]
    if (B.shape[0] if b_mn else B.shape[1]) != K:
        raise ValueError("inner dimensions differ")
    if out is None:
        if accumulate:
            raise ValueError("accumulate needs an out tensor")
        out = torch.empty((M, N), dtype=torch.bfloat16 if out_bf16 else torch.float32, device=A.device)
    mode = 2 if accumulate else (1 if out_bf16 else 0)
    check(lib().dt_gemm_bf16(A.data_ptr(), int(a_mn), B.data_ptr(), int(b_mn), out.data_ptr(), mode, M, N, K,
                             out.stride(0), _stream_ptr(A.device)))
    return out


def qk_norm_rope(q, k, v, q_gain, k_gain, B: int, T: int, eps: float = rms_eps, theta: float = rope_theta):
    """Prologue on fp32 rows (row stride taken from q): returns bf16 (q, k, v) [B*T, 2048]."""
    torch = _torch()
    M = B * T
    outs = [torch.empty((M, d_model), dtype=torch.bfloat16, device=q.device) for _ in range(3)]
    check(lib().dt_qk_norm_rope(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(0), q_gain.data_ptr(),
                                k_gain.data_ptr(), outs[0].data_ptr(), outs[1].data_ptr(), outs[2].data_ptr(), B, T,
                                float(eps), float(theta), _stream_ptr(q.device)))
    return tuple(outs)


def rope_tables(max_seq: int = max_seq_len, dim: int = head_dim, theta: float = rope_theta):
    """The RoPE sin/cos tables the device uses, as host arrays [max_seq, dim]."""
    s = np.empty((max_seq, dim), np.float32)
    c = np.empty((max_seq, dim), np.float32)
    check(lib().dt_rope_tables(s.ctypes.data, c.ctypes.data, max_seq, dim, float(theta)))
    return s, c


def check_device_error() -> None:
    """Synchronise the current device and raise if a kernel reported an expired wait."""
    check(lib().dt_check_device_error())


class OlmoAttention:
    """Drop-in for OlmoAttention (OlmoAttention.h:10-42): forward, backward, step, zero_grad.

    ``OlmoAttention(folder, index)`` loads the six ``.npy`` weight files of
    layer ``index`` as OlmoAttention.cpp:39-46 does; ``OlmoAttention.from_weights``
    takes arrays directly.  Weights live on ``device`` as bf16 (projections) and
    fp32 (norm gains).
    """

    def __init__(self, folder: Optional[str] = None, index: int = 0, device: int = 0, _handle=None):
        self._h = ctypes.c_void_p()
        self.device = device
        if _handle is not None:
            self._h = _handle
        elif folder is not None:
            check(lib().dt_attn_create_from_npy(folder.encode(), int(index), int(device), ctypes.byref(self._h)))
        else:
            raise ValueError("OlmoAttention needs a checkpoint folder (or use from_weights)")

    @classmethod
    def from_weights(cls, q_proj, k_proj, v_proj, o_proj, q_norm, k_norm, device: int = 0,
                     eps: float = rms_eps, theta: float = rope_theta) -> "OlmoAttention":
        arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (q_proj, k_proj, v_proj, o_proj, q_norm, k_norm)]
        for a in arrs[:4]:
            if a.shape != (d_model, d_model):
                raise ValueError(f"projection weights must be [{d_model}, {d_model}]")
        for a in arrs[4:]:
            if a.shape != (d_model,):
                raise ValueError(f"norm gains must be [{d_model}]")
        w = dt_attn_weights(*(a.ctypes.data for a in arrs), d_model, n_heads, eps, theta)
        h = ctypes.c_void_p()
        check(lib().dt_attn_create(ctypes.byref(w), int(device), ctypes.byref(h)))
        return cls(device=device, _handle=h)

    def forward(self, x, seq_lens=None, out=None):
        """x: [B, T, 2048] float32 (CUDA tensor or numpy).  seq_lens: optional
        per-sequence lengths for right-padded batches (rows past a sequence's
        length are returned as zeros)."""
        if _is_torch(x):
            torch = _torch()
            _need_cuda_f32("x", x, 3)
            B, T, _ = x.shape
            y = out if out is not None else torch.empty_like(x)
            lens = None
            if seq_lens is not None:
                lens = torch.as_tensor(seq_lens, dtype=torch.int32, device=x.device).contiguous()
            check(lib().dt_attn_forward(self._h, x.data_ptr(), B, T, _ptr(lens), y.data_ptr(),
                                        _stream_ptr(x.device)))
            return y
        x = np.ascontiguousarray(x, dtype=np.float32)
        B, T, _ = x.shape
        y = np.empty_like(x)
        lens_p = None
        if seq_lens is not None:
            lens = np.ascontiguousarray(seq_lens, dtype=np.int32)
            lens_p = lens.ctypes.data
        check(lib().dt_attn_forward_host(self._h, x.ctypes.data, B, T, lens_p, y.ctypes.data))
        return y

    __call__ = forward

    def backward(self, d_output, out=None):
        """OlmoAttention::backward (OlmoAttention.cpp:189-312): gradient of the
        last forward's input, given d_output [B, T, 2048] float32 of that
        forward's shape (a forward without seq_lens).  Weight gradients
        accumulate in the handle until zero_grad()."""
        if _is_torch(d_output):
            torch = _torch()
            _need_cuda_f32("d_output", d_output, 3)
            B, T, _ = d_output.shape
            dx = out if out is not None else torch.empty_like(d_output)
            check(lib().dt_attn_backward(self._h, d_output.data_ptr(), B, T, dx.data_ptr(),
                                         _stream_ptr(d_output.device)))
            return dx
        dy = np.ascontiguousarray(d_output, dtype=np.float32)
        B, T, _ = dy.shape
        dx = np.empty_like(dy)
        check(lib().dt_attn_backward_host(self._h, dy.ctypes.data, B, T, dx.ctypes.data))
        return dx

    def step(self, lr: float, stream=None):
        """SGD step w -= lr * grad on every parameter (OlmoAttention.cpp:315-322)."""
        check(lib().dt_attn_step(self._h, float(lr), stream))

    def zero_grad(self, stream=None):
        """Clears the accumulated gradients (OlmoAttention.cpp:324-330)."""
        check(lib().dt_attn_zero_grad(self._h, stream))

    def parameters(self, gradients: bool = False) -> dict:
        """Host copies of the fp32 weights (or of their gradients) keyed like the checkpoint."""
        d = d_model
        out = {k: np.empty((d, d), np.float32) for k in ("q_proj", "k_proj", "v_proj", "o_proj")}
        out.update({k: np.empty(d, np.float32) for k in ("q_norm", "k_norm")})
        check(lib().dt_attn_get_params_host(self._h, *(out[k].ctypes.data for k in
                                                      ("q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm")),
                                            int(gradients)))
        return out

    def close(self):
        if self._h:
            lib().dt_attn_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


LAYER_KEYS = ("q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm", "post_attention_norm", "gate_proj",
              "up_proj", "down_proj", "post_feedforward_norm")


class OlmoModel:
    """Full OLMo-2 prefill on the GPU: mirror of OlmoModel (OlmoModel.h:11-31),
    forward path.  ``OlmoModel(folder)`` reads the checkpoint as OlmoModel.cpp:11-22
    does; ``OlmoModel.from_weights`` takes arrays (a list of per-layer dicts with
    LAYER_KEYS).  ``forward(ids)`` returns logits [B, T, vocab] (fp32)."""

    def __init__(self, folder: Optional[str] = None, device: int = 0, n_layers: int = n_layers, _handle=None):
        self._h = ctypes.c_void_p()
        self.device = device
        if _handle is not None:
            self._h = _handle
        elif folder is not None:
            check(lib().dt_model_create_from_npy(folder.encode(), int(n_layers), int(device), ctypes.byref(self._h)))
        else:
            raise ValueError("OlmoModel needs a checkpoint folder (or use from_weights)")
        nl, voc, hid = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        check(lib().dt_model_info(self._h, ctypes.byref(nl), ctypes.byref(voc), ctypes.byref(hid)))
        self.n_layers, self.vocab, self.hidden = nl.value, voc.value, hid.value

    @classmethod
    def from_weights(cls, embed, layers, final_norm, lm_head, device: int = 0, eps: float = rms_eps,
                     theta: float = rope_theta) -> "OlmoModel":
        embed = np.ascontiguousarray(embed, dtype=np.float32)
        lm_head = np.ascontiguousarray(lm_head, dtype=np.float32)
        final_norm = np.ascontiguousarray(final_norm, dtype=np.float32)
        keep = [embed, lm_head, final_norm]
        arr = (dt_model_layer_weights * len(layers))()
        for i, lw in enumerate(layers):
            for k in LAYER_KEYS:
                a = np.ascontiguousarray(lw[k], dtype=np.float32)
                keep.append(a)
                setattr(arr[i], k, a.ctypes.data)
        hidden = int(np.asarray(layers[0]["up_proj"]).shape[0])
        w = dt_model_weights(embed.ctypes.data, final_norm.ctypes.data, lm_head.ctypes.data, arr, len(layers),
                             int(embed.shape[0]), d_model, n_heads, hidden, eps, theta)
        h = ctypes.c_void_p()
        check(lib().dt_model_create(ctypes.byref(w), int(device), ctypes.byref(h)))
        return cls(device=device, _handle=h)

    def forward(self, ids, out=None):
        """ids: [B, T] uint32/int token ids (CUDA tensor: device path; numpy: host path)."""
        if _is_torch(ids):
            torch = _torch()
            B, T = ids.shape
            t = ids.to(torch.int32).contiguous()
            logits = out if out is not None else torch.empty((B, T, self.vocab), dtype=torch.float32,
                                                             device=ids.device)
            check(lib().dt_model_forward(self._h, t.data_ptr(), B, T, logits.data_ptr(), _stream_ptr(ids.device)))
            return logits
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        B, T = ids.shape
        logits = np.empty((B, T, self.vocab), np.float32)
        check(lib().dt_model_forward_host(self._h, ids.ctypes.data, B, T, logits.ctypes.data))
        return logits

    __call__ = forward

    def close(self):
        if self._h:
            lib().dt_model_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
