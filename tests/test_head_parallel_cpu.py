"""CPU test (gloo, world_size 2 and 4) of the head-parallel host logic: head and
token ranges, the token-sliced all-to-all and the planar O-projection layout.
The per-rank compute steps are replaced by the CPU oracle so the exchange logic
runs without a GPU; the assembled token slices must equal the unsharded result."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from common import SCALE, qkv, randn


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, B, T, H, out_dir, exchange="nccl"):
    import torch.distributed as dist

    import oracle
    from dirktensor_b200.head_parallel import HeadParallelAttention, head_range, token_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)

    class CpuHeadParallel(HeadParallelAttention):
        def _prepare_wo(self, wo):
            return wo.contiguous()

        def local_attention(self, q, k, v, scale, causal, events=None):
            o, _, _ = oracle.flash_fwd(q.numpy(), k.numpy(), v.numpy(), scale, causal)
            Bq, Tq, Hl, D = q.shape
            return torch.from_numpy(o.reshape(Bq * Tq, Hl * D))

        def project(self, a, planes, out=None):
            A = a.permute(1, 0, 2).reshape(a.shape[1], -1) if planes > 1 else a
            y = torch.from_numpy(oracle.linear(A.contiguous().numpy(), self.wo.numpy()))
            if out is not None:
                out.copy_(y)
                return out
            return y

    q, k, v = qkv(5, B, T, H)
    wo = randn(6, (2048 // 16 * H, 2048 // 16 * H), 0.02)
    h0, h1 = head_range(rank, world, H)
    hp = CpuHeadParallel(torch.from_numpy(wo), n_heads=H, head_dim=128, exchange=exchange)
    y = hp.forward(*(torch.from_numpy(np.ascontiguousarray(a[:, :, h0:h1])) for a in (q, k, v)), SCALE, True)
    t0, t1 = token_range(rank, world, B * T) if exchange != "allgather" else (0, B * T)
    np.save(os.path.join(out_dir, f"y{rank}.npy"), y.numpy())
    np.save(os.path.join(out_dir, f"range{rank}.npy"), np.array([t0, t1]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,exchange", [(2, "nccl"), (4, "nccl"), (2, "allgather"), (4, "allgather")])
def test_head_parallel_exchange_matches_unsharded(tmp_path, world, exchange):
    """Token-sliced all-to-all: each rank gets its token slice; replicated
    all-gather: every rank gets the whole output."""
    import oracle

    B, T, H = 2, 96, 8
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, T, H, str(tmp_path), exchange))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    q, k, v = qkv(5, B, T, H)
    d = 128 * H
    wo = randn(6, (d, d), 0.02)
    o, _, _ = oracle.flash_fwd(q, k, v, SCALE, True)
    ref = oracle.linear(o.reshape(B * T, d), wo)
    for r in range(world):
        t0, t1 = np.load(tmp_path / f"range{r}.npy")
        y = np.load(tmp_path / f"y{r}.npy")
        assert y.shape == (t1 - t0, d)
        assert np.max(np.abs(y - ref[t0:t1])) < 1e-4


def test_ranges():
    from dirktensor_b200.head_parallel import head_range, token_range

    assert [head_range(r, 4, 16) for r in range(4)] == [(0, 4), (4, 8), (8, 12), (12, 16)]
    assert token_range(3, 8, 98304) == (36864, 49152)
    with pytest.raises(ValueError):
        head_range(0, 3, 16)
