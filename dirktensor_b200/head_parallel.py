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
Two exchange modes:
  fused (default): the flash kernel's epilogue
      stores each output row straight into the owning rank's receive buffer
      over NVLink (peer pointers from CUDA IPC, plain stores), i.e. attention and
      exchange are one kernel; a one-element all-reduce on the same stream then
      orders every rank's stores before the owners' O projections.  Receive
      buffers are double-buffered across steps, so a rank that runs ahead never
      overwrites a buffer its owner is still projecting.  Rows leave through
      shared memory so that each warp stores two whole 256-byte rows per
      instruction to the peer; one system-scope fence kernel after the
      attention kernel (not one fence per storing thread) publishes the stores.
      The attention kernel reads this rank's Q in fp32 and rounds it itself
      (K and V are cast first, in one launch).  Measured at 2 GPUs (config 4): 1.70 ms per
      step; 2.09 ms for the NCCL path.
  nccl: the flash kernel writes a local [M, Hl*D] buffer and
      torch.distributed.all_to_all_single moves the token slices.
The attention and projection kernels are the CUDA library's.
"""
from __future__ import annotations

from typing import Optional, Tuple

import ctypes

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
                 group: Optional[dist.ProcessGroup] = None, exchange: str = "fused"):
        if exchange not in ("fused", "nccl"):
            raise ValueError("exchange must be 'fused' or 'nccl'")
        self.exchange_mode = exchange
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.h0, self.h1 = head_range(self.rank, self.world, n_heads)
        self.wo = self._prepare_wo(wo)
        self._bufs = {}
        self._fused = None   # (shape, [recv buffers], [peer pointer arrays], [(ptr, offset) opened])
        self._step = 0

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
        kb, vb = _attn.cast2_bf16(k.contiguous(), v.contiguous())  # the attention kernel rounds q itself
        out = self._buf("o_local", (B * T, Hl * D), torch.bfloat16, q.device)
        if events is not None:
            events[0].record()
        _attn.flash_attention_forward_qf32(q.contiguous(), kb, vb, scale, causal, out=out, out_bf16=True,
                                           out_row_stride=Hl * D)
        if events is not None:
            events[1].record()
        return out

    def project(self, a: torch.Tensor, planes: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y = A . Wo^T for A planar over `planes` planes ([planes, m, K/planes]).
        `out` ([m, d] float32, contiguous) receives y; by default a buffer that
        the next call reuses."""
        m = a.shape[1] if planes > 1 else a.shape[0]
        d = self.wo.shape[0]
        if out is None:
            y = self._buf("y", (m, d), torch.float32, a.device)
        else:
            if out.shape != (m, d) or out.dtype != torch.float32 or not out.is_contiguous():
                raise ValueError(f"out must be a contiguous float32 [{m}, {d}] tensor")
            y = out
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

    # ---- fused attention + exchange ------------------------------------------
    def _setup_fused(self, M: int, w: int, device):
        """Two receive buffers [G, M/G, w] bf16 per rank; every rank maps every
        peer's buffers through CUDA IPC (64-byte handles all-gathered once)."""
        G = self.world
        shape = (G, M // G, w)
        if self._fused is not None and self._fused[0] == shape:
            return
        self.close()
        L = lib()
        recv = [torch.empty(shape, dtype=torch.bfloat16, device=device) for _ in range(2)]
        mine = torch.zeros((2, 72), dtype=torch.uint8)
        for i, buf in enumerate(recv):
            h = (ctypes.c_uint8 * 64)()
            off = ctypes.c_size_t()
            check(L.dt_ipc_get_handle(buf.data_ptr(), h, ctypes.byref(off)))
            mine[i, :64] = torch.tensor(list(bytes(h)), dtype=torch.uint8)
            mine[i, 64:] = torch.tensor(list(off.value.to_bytes(8, "little")), dtype=torch.uint8)
        allh = torch.empty((G, 2, 72), dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(allh, mine.to(device), group=self.group)
        allh = allh.cpu()
        ptrs, opened = [], []
        for i in range(2):
            arr = (ctypes.c_void_p * G)()
            for r in range(G):
                if r == self.rank:
                    arr[r] = recv[i].data_ptr()
                    continue
                hb = bytes(allh[r, i, :64].tolist())
                off = int.from_bytes(bytes(allh[r, i, 64:].tolist()), "little")
                p = ctypes.c_void_p()
                check(L.dt_ipc_open((ctypes.c_uint8 * 64).from_buffer_copy(hb), off, ctypes.byref(p)))
                arr[r] = p.value
                opened.append((p.value, off))
            ptrs.append(arr)
        self._fused = (shape, recv, ptrs, opened)
        self._barrier = torch.zeros(1, dtype=torch.float32, device=device)

    def close(self):
        """Unmaps the peers' receive buffers (fused exchange)."""
        if self._fused is not None:
            for ptr, off in self._fused[3]:
                lib().dt_ipc_close(ctypes.c_void_p(ptr), off)
            self._fused = None

    def fused_attention_exchange(self, q, k, v, scale: float, causal: bool, events=None) -> torch.Tensor:
        """One kernel computes this rank's heads and stores every output row in
        its owner's receive buffer; returns this rank's filled receive buffer."""
        B, T, Hl, D = q.shape
        M = B * T
        self._setup_fused(M, Hl * D, q.device)
        buf = self._step & 1
        self._step += 1
        kb, vb = _attn.cast2_bf16(k.contiguous(), v.contiguous())  # the attention kernel rounds q itself
        q = q.contiguous()
        if events is not None:
            events[0].record()
        check(lib().dt_flash_fwd_qf32_exchange(q.data_ptr(), kb.data_ptr(), vb.data_ptr(), self._fused[2][buf],
                                               self.world, self.rank, M // self.world, None, None, B, T, Hl, D,
                                               float(scale), int(bool(causal)),
                                               torch.cuda.current_stream(q.device).cuda_stream))
        if events is not None:
            events[1].record()
        # stream-ordered barrier: every rank's stores into my buffer precede my projection
        dist.all_reduce(self._barrier, group=self.group)
        return self._fused[1][buf]

    def forward(self, q, k, v, scale: float, causal: bool = True, events=None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        B, T, Hl, D = q.shape
        if Hl != self.h1 - self.h0 or D != self.head_dim:
            raise ValueError(f"expected [B, T, {self.h1 - self.h0}, {self.head_dim}] local heads")
        token_range(self.rank, self.world, B * T)  # validates divisibility
        if self.world > 1 and self.exchange_mode == "fused" and q.is_cuda:
            a = self.fused_attention_exchange(q, k, v, scale, causal, events)
        else:
            o_local = self.local_attention(q, k, v, scale, causal, events)
            a = self.exchange(o_local)
        return self.project(a, self.world, out)

    __call__ = forward
