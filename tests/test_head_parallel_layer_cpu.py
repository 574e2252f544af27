"""CPU test (gloo, world_size 2 and 4) of the head-parallel attention LAYER's
host logic (HeadParallelAttentionLayer): column-parallel Q/K/V rows of each
rank's heads, the per-token sums of squares all-reduced over the ranks (the
QK-RMSNorm normalises over all 2048 columns, RMSNorm.cpp:17, across heads),
the gains sliced per rank, RoPE per local head, the token-sliced all-to-all
and the planar O projection.  Each rank's compute steps are replaced by the
CPU oracle (fp32), so the sharding runs without a GPU.  The assembled token
slices must equal the oracle's unsharded OlmoAttention::forward
(OlmoAttention.cpp:56-108) of the full 16-head layer, on a square batch and on
a right-padded (varlen) batch."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from common import SCALE, layer_weights

EPS = 1e-6


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(B, T):
    x = np.random.default_rng(17).standard_normal((B, T, 2048), dtype=np.float32)
    return x, layer_weights(31)


def _worker(rank, world, port, B, T, lens, out_dir):
    import torch.distributed as dist

    import oracle
    from dirktensor_b200.head_parallel import HeadParallelAttentionLayer, token_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)

    class CpuLayer(HeadParallelAttentionLayer):
        def _prepare_wo(self, wo):
            return wo.contiguous()

        def _prepare_wqkv(self, w):
            return w.contiguous()

        def project_qkv(self, x2d):
            return torch.from_numpy(oracle.linear(x2d.contiguous().numpy(), self.wqkv.numpy()))

        def sums_of_squares(self, qkv):
            w = self.width
            q, k = qkv[:, :w].double(), qkv[:, w:2 * w].double()
            return torch.stack([(q * q).sum(1), (k * k).sum(1)], 1).float()

        def norm_rope(self, qkv, ss, B, T):
            w = self.width
            Hl = w // 128
            rq = torch.sqrt(ss[:, 0:1] / 2048.0 + EPS)
            rk = torch.sqrt(ss[:, 1:2] / 2048.0 + EPS)
            qn = (qkv[:, :w] / rq * self.q_gain).reshape(B, T, Hl, 128).numpy()
            kn = (qkv[:, w:2 * w] / rk * self.k_gain).reshape(B, T, Hl, 128).numpy()
            v = qkv[:, 2 * w:].reshape(B, T, Hl, 128).contiguous()
            return torch.from_numpy(oracle.rope(qn)), torch.from_numpy(oracle.rope(kn)), v

        def attention_bf16(self, q, k, v, seq_lens):
            B, T, Hl, D = q.shape
            o, _, _ = oracle.flash_fwd(q.numpy(), k.numpy(), v.numpy(), SCALE, True)
            if seq_lens is not None:
                for b, n in enumerate(seq_lens):
                    o[b, n:] = 0.0
            return self.exchange(torch.from_numpy(o.reshape(B * T, Hl * D)))

        def project(self, a, planes, out=None):
            A = a.permute(1, 0, 2).reshape(a.shape[1], -1) if planes > 1 else a
            return torch.from_numpy(oracle.linear(A.contiguous().numpy(), self.wo.numpy()))

    x, (wq, wk, wv, wo, qg, kg) = _inputs(B, T)
    t = [torch.from_numpy(a) for a in (wq, wk, wv, wo, qg, kg)]
    layer = CpuLayer(*t, exchange="nccl")
    y = layer.forward(torch.from_numpy(x), seq_lens=lens)
    t0, t1 = token_range(rank, world, B * T)
    np.save(os.path.join(out_dir, f"y{rank}.npy"), y.numpy())
    np.save(os.path.join(out_dir, f"range{rank}.npy"), np.array([t0, t1]))
    dist.barrier()
    dist.destroy_process_group()


def _run(tmp_path, world, B, T, lens):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, T, lens, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    y = np.zeros((B * T, 2048), np.float32)
    for r in range(world):
        t0, t1 = np.load(tmp_path / f"range{r}.npy")
        ys = np.load(tmp_path / f"y{r}.npy")
        assert ys.shape == (t1 - t0, 2048)
        y[t0:t1] = ys
    return y.reshape(B, T, 2048)


@pytest.mark.parametrize("world", [2, 4])
def test_layer_head_parallel_matches_unsharded(tmp_path, world):
    import oracle

    B, T = 2, 96
    y = _run(tmp_path, world, B, T, None)
    x, w = _inputs(B, T)
    ref = oracle.attention_layer(x, *w)
    err = float(np.linalg.norm(y - ref) / np.linalg.norm(ref))
    assert err < 1e-5, err


@pytest.mark.parametrize("world", [2, 4])
def test_layer_head_parallel_varlen_matches_per_sequence(tmp_path, world):
    import oracle

    B, T, lens = 2, 96, [61, 96]
    y = _run(tmp_path, world, B, T, lens)
    x, w = _inputs(B, T)
    for b, n in enumerate(lens):
        ref = oracle.attention_layer(x[b:b + 1, :n], *w)[0]
        err = float(np.linalg.norm(y[b, :n] - ref) / np.linalg.norm(ref))
        assert err < 1e-5, (b, err)
        assert not np.any(y[b, n:])
