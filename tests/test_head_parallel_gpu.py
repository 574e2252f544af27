"""GPU tests of the head-parallel path (attention + token-sliced exchange + planar
O projection).  World size 1 runs on any single GPU; world size 2 runs as child
processes over NCCL when two GPUs are visible (skipped otherwise)."""
import os
import socket

import numpy as np
import pytest

import oracle
from common import SCALE, qkv, randn, rel_l2

pytestmark = pytest.mark.gpu

B, T, H = 2, 640, 16


def _reference(B, T, H):
    q, k, v = qkv(55, B, T, H)
    wo = randn(56, (2048, 2048), 0.02)
    o, _, _ = oracle.flash_fwd(q, k, v, SCALE, True)
    return q, k, v, wo, oracle.linear(o.reshape(B * T, 2048), wo)


def _run_rank(rank, world, q, k, v, wo, exchange="fused", steps=1):
    import torch

    from dirktensor_b200.head_parallel import HeadParallelAttention, head_range

    dev = torch.device("cuda", rank)
    h0, h1 = head_range(rank, world, H)
    hp = HeadParallelAttention(torch.from_numpy(wo).to(dev), n_heads=H, head_dim=128, exchange=exchange)
    ql, kl, vl = (torch.from_numpy(np.ascontiguousarray(a[:, :, h0:h1])).to(dev) for a in (q, k, v))
    ys = []
    for _ in range(steps):  # several steps exercise both receive buffers
        ys.append(hp.forward(ql, kl, vl, SCALE, True).cpu().numpy())
    torch.cuda.synchronize(dev)
    hp.close()
    for y in ys[1:]:
        assert np.array_equal(y, ys[0])
    return ys[0]


def test_head_parallel_world1_vs_oracle(cuda):
    import dirktensor_b200 as dt

    q, k, v, wo, ref = _reference(B, T, H)
    y = _run_rank(0, 1, q, k, v, wo)
    dt.check_device_error()
    assert rel_l2(y, ref) < 1.5e-2


def test_planar_gemm_equals_plain_gemm_on_concatenated_planes(cuda):
    import torch

    import dirktensor_b200 as dt
    from dirktensor_b200._lib import check, lib

    G, m, w, N = 4, 300, 256, 512
    planes = torch.from_numpy(randn(3, (G, m, w))).to(cuda).to(torch.bfloat16)
    wo = torch.from_numpy(randn(4, (N, G * w), 0.05)).to(cuda).to(torch.bfloat16)
    y = torch.empty((m, N), device=cuda)
    check(lib().dt_gemm_bf16_tn_planar(planes.data_ptr(), G, wo.data_ptr(), y.data_ptr(), 0, m, N, G * w, N,
                                       torch.cuda.current_stream().cuda_stream))
    a = planes.permute(1, 0, 2).reshape(m, G * w).contiguous()
    y2 = dt.gemm_bf16_tn(a, wo)
    dt.check_device_error()
    assert torch.equal(y, y2)


def _worker(rank, world, port, out_dir, exchange):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    q, k, v, wo, _ = _reference(B, T, H)
    y = _run_rank(rank, world, q, k, v, wo, exchange=exchange, steps=3)
    np.save(os.path.join(out_dir, f"y{rank}.npy"), y)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["fused", "nccl"])
def test_head_parallel_world2(cuda, tmp_path, exchange):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path), exchange)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    _, _, _, _, ref = _reference(B, T, H)
    M = B * T
    for r in range(2):
        y = np.load(tmp_path / f"y{r}.npy")
        assert rel_l2(y, ref[r * M // 2:(r + 1) * M // 2]) < 1.5e-2
