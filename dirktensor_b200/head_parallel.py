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
      exchange are one kernel; a flag barrier kernel on the same stream (each
      rank releases a step counter into every rank's flag array over NVLink and
      waits, bounded, for all of them) then orders every rank's stores before
      the owners' O projections.  Receive
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
  allgather: the replicated form -- an all-gather of every rank's per-head
      outputs ((G-1)/G of the output into every rank), then every rank projects
      all B*T tokens.  Kept to measure against the token-sliced forms.
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
        if exchange not in ("fused", "nccl", "allgather"):
            raise ValueError("exchange must be 'fused', 'nccl' or 'allgather'")
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
        """[M, Hl*D] token-major -> [G, M/G, Hl*D]: plane g = rank g's heads of my tokens.
        With exchange 'allgather': -> [G, M, Hl*D], every rank's heads of every token."""
        G = self.world
        M, w = o_local.shape
        if G == 1:
            return o_local
        if self.exchange_mode == "allgather":
            full = self._buf("gathered", (G * M, w), o_local.dtype, o_local.device)
            dist.all_gather_into_tensor(full, o_local.contiguous(), group=self.group)
            return full.view(G, M, w)
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
        # the barrier's flag array (8 counters) travels with the receive buffers
        flags = torch.zeros(64, dtype=torch.int32, device=device)
        bufs = recv + [flags]
        mine = torch.zeros((3, 72), dtype=torch.uint8)
        for i, buf in enumerate(bufs):
            h = (ctypes.c_uint8 * 64)()
            off = ctypes.c_size_t()
            check(L.dt_ipc_get_handle(buf.data_ptr(), h, ctypes.byref(off)))
            mine[i, :64] = torch.tensor(list(bytes(h)), dtype=torch.uint8)
            mine[i, 64:] = torch.tensor(list(off.value.to_bytes(8, "little")), dtype=torch.uint8)
        allh = torch.empty((G * 3, 72), dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(allh, mine.to(device), group=self.group)
        allh = allh.view(G, 3, 72).cpu()
        ptrs, opened = [], []
        for i in range(3):
            arr = (ctypes.c_void_p * G)()
            for r in range(G):
                if r == self.rank:
                    arr[r] = bufs[i].data_ptr()
                    continue
                hb = bytes(allh[r, i, :64].tolist())
                off = int.from_bytes(bytes(allh[r, i, 64:].tolist()), "little")
                p = ctypes.c_void_p()
                check(L.dt_ipc_open((ctypes.c_uint8 * 64).from_buffer_copy(hb), off, ctypes.byref(p)))
                arr[r] = p.value
                opened.append((p.value, off))
            ptrs.append(arr)
        self._fused = (shape, recv, ptrs, opened, flags)

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
        # every rank's stores into my buffer precede my projection: flag barrier on the GPU
        check(lib().dt_exchange_barrier(self._fused[2][2], self.world, self.rank, self._step,
                                        torch.cuda.current_stream(q.device).cuda_stream))
        return self._fused[1][buf]

    def forward(self, q, k, v, scale: float, causal: bool = True, events=None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """This rank's token slice of y ([B*T/G, d]); with exchange 'allgather'
        (the replicated form: every rank gathers every head of every token and
        projects all B*T tokens) the whole y ([B*T, d]) on every rank."""
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


# ---------------------------------------------------------------------------
# The full attention layer, head-parallel
# ---------------------------------------------------------------------------
class HeadParallelAttentionLayer(HeadParallelAttention):
    """OlmoAttention::forward (OlmoAttention.cpp:56-108) with the heads sharded
    over the process group, orchestrated with torch.distributed:

      [q|k|v]_r = x [Wq_r; Wk_r; Wv_r]^T   column-parallel: rank r's head rows
      s_r = per-token sums of squares of q_r and k_r, all-reduced: QK-RMSNorm
            normalises over all 2048 columns (RMSNorm.cpp:17), i.e. over every
            rank's heads, so 2 floats per token cross the ranks
      q_r, k_r = RoPE(q_r / rms * g_r); v_r     this rank's heads only
      attention + token-sliced exchange + O projection of HeadParallelAttention.

    ``forward(x)`` takes the full input [B, T, 2048] float32 on every rank and
    returns this rank's token slice of y ([B*T/G, 2048]).  The same
    orchestration for C/C++ callers is ShardedOlmoAttention (the C ABI's
    dt_attn_create_sharded / dt_attn_forward_sharded, on a communicator of its
    own).  The compute steps are methods so that host tests can replace them.
    """

    def __init__(self, wq, wk, wv, wo, q_norm, k_norm, group: Optional[dist.ProcessGroup] = None,
                 exchange: str = "fused", eps: float = 1e-6, theta: float = 500000.0):
        super().__init__(wo, n_heads=16, head_dim=128, group=group, exchange=exchange)
        rows = slice(self.h0 * self.head_dim, self.h1 * self.head_dim)
        self.width = (self.h1 - self.h0) * self.head_dim
        self.wqkv = self._prepare_wqkv(torch.cat([wq[rows], wk[rows], wv[rows]]).contiguous())
        self.q_gain = q_norm[rows].contiguous()
        self.k_gain = k_norm[rows].contiguous()
        self.eps = eps
        self.theta = theta

    # ---- compute steps (CUDA library) ------------------------------------
    def _prepare_wqkv(self, w):
        return _attn.cast_bf16(w)

    def project_qkv(self, x2d):
        """[M, 2048] float32 -> [M, 3w] float32 (this rank's q, k, v columns)."""
        return _attn.gemm_bf16_tn(_attn.cast_bf16(x2d.contiguous()), self.wqkv)

    def sums_of_squares(self, qkv):
        """Per-token {sum q^2, sum k^2} over this rank's columns: [M, 2] float32."""
        M = qkv.shape[0]
        ss = torch.empty((M, 2), dtype=torch.float32, device=qkv.device)
        w = self.width
        check(lib().dt_qk_sumsq(qkv.data_ptr(), qkv[:, w:].data_ptr(), qkv.stride(0), w, M, ss.data_ptr(),
                                torch.cuda.current_stream(qkv.device).cuda_stream))
        return ss

    def norm_rope(self, qkv, ss, B: int, T: int):
        """q, k normalised with the full-row sums and RoPE'd, v copied: bf16 [B, T, Hl, D] each."""
        M, w = qkv.shape[0], self.width
        Hl = self.h1 - self.h0
        outs = [torch.empty((B, T, Hl, self.head_dim), dtype=torch.bfloat16, device=qkv.device) for _ in range(3)]
        check(lib().dt_qk_norm_rope_shard(qkv.data_ptr(), qkv[:, w:].data_ptr(), qkv[:, 2 * w:].data_ptr(),
                                          qkv.stride(0), ss.data_ptr(), self.q_gain.data_ptr(),
                                          self.k_gain.data_ptr(), Hl, outs[0].data_ptr(), outs[1].data_ptr(),
                                          outs[2].data_ptr(), B, T, float(self.eps), float(self.theta),
                                          torch.cuda.current_stream(qkv.device).cuda_stream))
        return tuple(outs)

    def attention_bf16(self, qb, kb, vb, seq_lens):
        """Attention on this rank's heads (bf16 operands) -> the A operand of the
        O projection: [M, w] (one rank) or [G, M/G, w] (after the exchange)."""
        B, T, Hl, D = qb.shape
        M = B * T
        G = self.world
        scale = 1.0 / float(D) ** 0.5
        lens = None if seq_lens is None else torch.as_tensor(seq_lens, dtype=torch.int32,
                                                             device=qb.device).contiguous()
        stream = torch.cuda.current_stream(qb.device).cuda_stream
        if G > 1 and self.exchange_mode == "fused":
            if lens is not None:
                raise ValueError("the in-kernel exchange of this Python layer takes no seq_lens; "
                                 "use exchange='nccl' or ShardedOlmoAttention")
            self._setup_fused(M, Hl * D, qb.device)
            buf = self._step & 1
            self._step += 1
            check(lib().dt_flash_fwd_bf16_exchange(qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), self._fused[2][buf],
                                                   G, self.rank, M // G, None, None, B, T, Hl, D, scale, 1, stream))
            check(lib().dt_exchange_barrier(self._fused[2][2], G, self.rank, self._step, stream))
            return self._fused[1][buf]
        out = self._buf("o_local", (M, Hl * D), torch.bfloat16, qb.device)
        check(lib().dt_flash_fwd_bf16(qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), out.data_ptr(), 1, Hl * D, None,
                                      None, None if lens is None else lens.data_ptr(), B, T, Hl, D, scale, 1,
                                      stream))
        return self.exchange(out)

    def forward(self, x, seq_lens=None, out: Optional[torch.Tensor] = None):  # type: ignore[override]
        B, T, d = x.shape
        M = B * T
        token_range(self.rank, self.world, M)  # validates divisibility
        qkv = self.project_qkv(x.reshape(M, d))
        ss = self.sums_of_squares(qkv)
        if self.world > 1:
            dist.all_reduce(ss, group=self.group)
        qb, kb, vb = self.norm_rope(qkv, ss, B, T)
        a = self.attention_bf16(qb, kb, vb, seq_lens)
        return self.project(a, self.world, out)

    __call__ = forward


class Communicator:
    """An NCCL communicator of the CUDA library (dt_comm) for this rank.

    ``Communicator.from_process_group()`` makes rank 0's 128-byte NCCL id
    (dt_comm_unique_id), hands it to the other ranks through torch.distributed
    (any backend), and creates the communicator on the current CUDA device with
    a set-up timeout (a rank that never joins makes the others fail with
    DT_ERR_TIMEOUT instead of hanging)."""

    def __init__(self, world: int, rank: int, uid: bytes, device: int, timeout_ms: int = 60000):
        self._c = ctypes.c_void_p()
        self.world, self.rank, self.device = world, rank, device
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
        check(lib().dt_comm_create(buf, world, rank, device, int(timeout_ms), ctypes.byref(self._c)))

    @staticmethod
    def unique_id() -> bytes:
        buf = (ctypes.c_uint8 * 128)()
        check(lib().dt_comm_unique_id(buf))
        return bytes(buf)

    @classmethod
    def from_process_group(cls, group: Optional[dist.ProcessGroup] = None, device: Optional[int] = None,
                           timeout_ms: int = 60000) -> "Communicator":
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        rank = dist.get_rank(group) if dist.is_initialized() else 0
        dev = torch.cuda.current_device() if device is None else device
        uid = cls.unique_id() if rank == 0 else bytes(128)
        if world > 1:
            backend = dist.get_backend(group)
            t = torch.tensor(list(uid), dtype=torch.uint8,
                             device=torch.device("cuda", dev) if backend == "nccl" else "cpu")
            dist.broadcast(t, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
            uid = bytes(t.cpu().tolist())
        return cls(world, rank, uid, dev, timeout_ms)

    @property
    def handle(self):
        return self._c

    def abort(self):
        if self._c:
            check(lib().dt_comm_abort(self._c))

    def close(self):
        if self._c:
            check(lib().dt_comm_destroy(self._c))
            self._c = ctypes.c_void_p()


class ShardedOlmoAttention:
    """The head-parallel attention layer of the C ABI (dt_attn_create_sharded,
    dt_attn_forward_sharded): the same steps as HeadParallelAttentionLayer, with
    the collectives issued by the library on its own NCCL communicator, so that
    C and C++ callers need no Python.  ``forward(x)`` takes the full input
    [B, T, 2048] float32 on every rank and returns this rank's token slice of y
    ([B*T/G, 2048]); exchange "fused" = in-kernel NVLink stores, "nccl" = NCCL
    all-to-all."""

    def __init__(self, wq, wk, wv, wo, q_norm, k_norm, comm: Communicator, exchange: str = "fused",
                 eps: float = 1e-6, theta: float = 500000.0):
        import numpy as np

        if exchange not in ("fused", "nccl"):
            raise ValueError("exchange must be 'fused' or 'nccl'")
        arrs = [np.ascontiguousarray(a.cpu().numpy() if hasattr(a, "cpu") else a, dtype=np.float32)
                for a in (wq, wk, wv, wo, q_norm, k_norm)]
        w = _attn.dt_attn_weights(*(a.ctypes.data for a in arrs), 2048, 16, eps, theta)
        self._h = ctypes.c_void_p()
        self.comm = comm
        check(lib().dt_attn_create_sharded(ctypes.byref(w), comm.handle, 0 if exchange == "fused" else 1,
                                           ctypes.byref(self._h)))

    def forward(self, x, seq_lens=None, out: Optional[torch.Tensor] = None, gather: bool = False):
        """gather=False: this rank's token slice [B*T/G, 2048]; gather=True: the
        whole output [B, T, 2048] on every rank."""
        B, T, d = x.shape
        G = self.comm.world
        if (B * T) % G:
            raise ValueError(f"B*T = {B * T} is not divisible by {G} ranks")
        shape = (B, T, d) if gather else (B * T // G, d)
        y = out if out is not None else torch.empty(shape, dtype=torch.float32, device=x.device)
        lens = None
        if seq_lens is not None:
            lens = torch.as_tensor(seq_lens, dtype=torch.int32, device=x.device).contiguous()
        check(lib().dt_attn_forward_sharded(self._h, x.contiguous().data_ptr(), B, T,
                                            None if lens is None else lens.data_ptr(), int(bool(gather)),
                                            y.data_ptr(), torch.cuda.current_stream(x.device).cuda_stream))
        return y

    __call__ = forward

    def close(self):
        if self._h:
            lib().dt_attn_destroy(self._h)
            self._h = ctypes.c_void_p()
