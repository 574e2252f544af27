"""Head-parallel attention over the ranks of one node (one process per GPU).

Attention for one (batch, head) pair needs no other head (FlashAttention.cpp
parallelises over B*H, :43-45), so the H heads are split into contiguous
blocks: rank r owns heads [r*H/G, (r+1)*H/G) of Q, K, V for all B*T tokens.
The O projection (OlmoAttention.cpp:99-107) mixes all heads of a token, so the
per-head outputs are exchanged once, token-sliced: rank r receives, from every
rank, that rank's heads for tokens [r*M/G, (r+1)*M/G) (M = B*T).  One
all-to-all moves (G-1)/G^2 of the output per rank (instead of (G-1)/G for a
replicated all-gather), and each rank then projects only its own token slice.

Layouts:
  local output   [M, Hl*D] bf16, token-major = [G, M/G, Hl*D] (chunk g -> rank g)
  received       [G, M/G, Hl*D] bf16 (plane g = rank g's heads)
  O projection   y[M/G, d] = A . Wo^T with A planar over G planes (plane g holds
                 columns [g*Hl*D, (g+1)*Hl*D) of the concatenated heads)
The exchange runs through torch.distributed (NCCL on GPUs); the attention and
projection kernels are the CUDA library's.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist

from . import attention as _attn
from ._lib import check, lib


def head_range(rank: int, world: int, n_heads: int) -> Tuple[int, int]:
    if n_heads % world:
        raise ValueError(f"{n_heads} heads do not split over {world} ranks")
    per = n_heads // world
    return rank * per, (rank + 1) * per


def token_range(rank: int, world: int, n_tokens: int) -> Tuple[int, int]:
    if n_tokens % world:
        raise ValueError(f"{n_tokens} tokens do not split over {world} ranks")
    per = n_tokens // world
    return rank * per, (rank + 1) * per


class HeadParallelAttention:
    """Attention + O projection with heads sharded over the process group.

    ``forward(q, k, v)`` takes this rank's heads ([B, T, H/G, D] float32) and
    returns this rank's token slice of y = attn . Wo^T ([B*T/G, d] float32).
    """

    exchange_dtype = torch.bfloat16

    def __init__(self, wo: torch.Tensor, n_heads: int = 16, head_dim: int = 128,
                 group: Optional[dist.ProcessGroup] = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.h0, self.h1 = head_range(self.rank, self.world, n_heads)
        self.wo = self._prepare_wo(wo)
        self._bufs = {}

    # ---- compute steps (CUDA library) ------------------------------------
    def _prepare_wo(self, wo: torch.Tensor) -> torch.Tensor:
        return _attn.cast_bf16(wo.contiguous())

    def _buf(self, name, shape, dtype, device):
        b = self._bufs.get(name)
        if b is None or b.shape != torch.Size(shape) or b.dtype != dtype or b.device != device:
            b = torch.empty(shape, dtype=dtype, device=device)
            self._bufs[name] = b
        return b

    def local_attention(self, q, k, v, scale: float, causal: bool, events=None) -> torch.Tensor:
        """Flash attention on this rank's heads -> bf16 [M, Hl*D]."""
        B, T, Hl, D = q.shape
        qb, kb, vb = (_attn.cast_bf16(t) for t in (q, k, v))
        out = self._buf("o_local", (B * T, Hl * D), torch.bfloat16, q.device)
        if events is not None:
            events[0].record()
        _attn.flash_attention_forward_bf16(qb, kb, vb, scale, causal, out=out, out_bf16=True,
                                           out_row_stride=Hl * D)
        if events is not None:
            events[1].record()
        return out

    def project(self, a: torch.Tensor, planes: int) -> torch.Tensor:
        """y = A . Wo^T for A planar over `planes` planes ([planes, m, K/planes])."""
        m = a.shape[1] if planes > 1 else a.shape[0]
        d = self.wo.shape[0]
        y = self._buf("y", (m, d), torch.float32, a.device)
        K = self.wo.shape[1]
        stream = torch.cuda.current_stream(a.device).cuda_stream
        if planes > 1:
            check(lib().dt_gemm_bf16_tn_planar(a.data_ptr(), planes, self.wo.data_ptr(), y.data_ptr(), 0, m, d, K,
                                               d, stream))
        else:
            check(lib().dt_gemm_bf16_tn(a.data_ptr(), self.wo.data_ptr(), y.data_ptr(), 0, m, d, K, d, stream))
        return y

    # ---- exchange ----------------------------------------------------------
    def exchange(self, o_local: torch.Tensor) -> torch.Tensor:
        """[M, Hl*D] token-major -> [G, M/G, Hl*D]: plane g = rank g's heads of my tokens."""
        G = self.world
        M, w = o_local.shape
        if G == 1:
            return o_local
        send = o_local.view(G, M // G, w)
        recv = self._buf("recv", (G, M // G, w), o_local.dtype, o_local.device)
        dist.all_to_all_single(recv, send, group=self.group)
        return recv

    def forward(self, q, k, v, scale: float, causal: bool = True, events=None) -> torch.Tensor:
        B, T, Hl, D = q.shape
        if Hl != self.h1 - self.h0 or D != self.head_dim:
            raise ValueError(f"expected [B, T, {self.h1 - self.h0}, {self.head_dim}] local heads")
        token_range(self.rank, self.world, B * T)  # validates divisibility
        o_local = self.local_attention(q, k, v, scale, causal, events)
        a = self.exchange(o_local)
        return self.project(a, self.world)

    __call__ = forward
