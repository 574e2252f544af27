"""GPU tests of the head-parallel attention LAYER (OlmoAttention::forward,
OlmoAttention.cpp:56-108, with the heads split over ranks): the C ABI's
dt_attn_create_sharded / dt_attn_forward_sharded on the library's own NCCL
communicator (ShardedOlmoAttention), and the torch.distributed orchestration
HeadParallelAttentionLayer.  Reference: the oracle's unsharded layer, on
configuration 0 (B=1, T=512) and a configuration-2 style right-padded batch
(valid rows against each sequence alone, padded rows zero).  World size 1 runs
on one GPU; world size 2 runs as child processes when two GPUs are visible."""
import datetime
import os
import socket

import numpy as np
import pytest

import oracle
from common import layer_weights, rel_l2

pytestmark = pytest.mark.gpu

TOL = 1.5e-2  # layer output, relative L2 (bf16 operands, fp32 accumulation)
CASES = {
    "config0": (1, 512, None),
    "varlen": (4, 1024, [1024, 333, 769, 128]),
}


def _inputs(case):
    B, T, lens = CASES[case]
    x = np.random.default_rng(11).standard_normal((B, T, 2048), dtype=np.float32)
    return x, layer_weights(12), lens


def _check(case, y_full):
    x, w, lens = _inputs(case)
    B, T, _ = x.shape
    y_full = y_full.reshape(B, T, 2048)
    if lens is None:
        ref = oracle.attention_layer(x, *w)
        assert rel_l2(y_full, ref) < TOL
        return
    for b, n in enumerate(lens):
        ref = oracle.attention_layer(x[b:b + 1, :n], *w)[0]
        assert rel_l2(y_full[b, :n], ref) < TOL, b
        assert not np.any(y_full[b, n:])


def _sharded(rank, world, dev, case, exchange, comm, gather=False):
    import torch

    from dirktensor_b200.head_parallel import ShardedOlmoAttention

    x, w, lens = _inputs(case)
    layer = ShardedOlmoAttention(*w, comm=comm, exchange=exchange)
    xd = torch.from_numpy(x).to(dev)
    ys = [layer.forward(xd, seq_lens=lens, gather=gather).cpu().numpy() for _ in range(3)]  # both receive buffers
    torch.cuda.synchronize(dev)
    layer.close()
    for y in ys[1:]:
        assert np.array_equal(y, ys[0])
    return ys[0]


@pytest.mark.parametrize("case", ["config0", "varlen"])
def test_sharded_layer_world1_vs_oracle(cuda, case):
    import dirktensor_b200 as dt
    from dirktensor_b200.head_parallel import Communicator

    comm = Communicator(1, 0, Communicator.unique_id(), 0, timeout_ms=60000)
    try:
        y = _sharded(0, 1, cuda, case, "fused", comm, gather=(case == "varlen"))
    finally:
        comm.close()
    dt.check_device_error()
    _check(case, y)


def test_sharded_layer_rejected_by_single_gpu_calls(cuda):
    import torch

    import dirktensor_b200 as dt
    from dirktensor_b200._lib import lib
    from dirktensor_b200.head_parallel import Communicator, ShardedOlmoAttention

    comm = Communicator(1, 0, Communicator.unique_id(), 0)
    x, w, _ = _inputs("config0")
    layer = ShardedOlmoAttention(*w, comm=comm)
    xd = torch.from_numpy(x).to(cuda)
    st = lib().dt_attn_forward(layer._h, xd.data_ptr(), 1, 512, None, xd.data_ptr(), None)
    assert st == 4 and b"sharded" in lib().dt_last_error()
    layer.close()
    comm.close()
    dt.check_device_error()


def _worker(rank, world, port, out_dir, impl, case, exchange, gather=False):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    if impl == "capi":
        from dirktensor_b200.head_parallel import Communicator

        comm = Communicator.from_process_group(timeout_ms=60000)
        y = _sharded(rank, world, dev, case, exchange, comm, gather)
        comm.close()
    else:
        from dirktensor_b200.head_parallel import HeadParallelAttentionLayer

        x, w, lens = _inputs(case)
        layer = HeadParallelAttentionLayer(*(torch.from_numpy(a).to(dev) for a in w), exchange=exchange)
        ys = [layer.forward(torch.from_numpy(x).to(dev), seq_lens=lens).cpu().numpy() for _ in range(3)]
        torch.cuda.synchronize(dev)
        layer.close()
        for yy in ys[1:]:
            assert np.array_equal(yy, ys[0])
        y = ys[0]
    np.save(os.path.join(out_dir, f"y{rank}.npy"), y)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("impl,case,exchange,gather", [("capi", "config0", "fused", False),
                                                       ("capi", "varlen", "fused", True),
                                                       ("capi", "varlen", "nccl", False),
                                                       ("torch", "config0", "fused", False),
                                                       ("torch", "varlen", "nccl", False)])
def test_sharded_layer_world2(cuda, tmp_path, impl, case, exchange, gather):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path), impl, case, exchange, gather))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    if gather:  # every rank holds the whole output
        for r in range(2):
            _check(case, np.load(tmp_path / f"y{r}.npy"))
    else:
        _check(case, np.concatenate([np.load(tmp_path / f"y{r}.npy") for r in range(2)]))
