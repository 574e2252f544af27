"""GPU test of the C++ drop-in (FlashAttention.h / OlmoAttention.h over the C ABI),
compiled with g++ the way a DirkTensor build would compile it, and driven the way
the reference's callers use it (OlmoAttention.cpp:94, OlmoBlock.cpp:6,14)."""
import os
import subprocess

import numpy as np
import pytest

import oracle
from common import (SCALE, TOL_ATTN_REL_L2, TOL_BWD_REL_L2, TOL_LAYER_BWD_REL_L2, TOL_LAYER_REL_L2,
                    layer_weights, qkv, randn, rel_l2)

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CPP = os.path.join(ROOT, "dirktensor_b200", "cpp")


@pytest.fixture(scope="module")
def dropin_bin(tmp_path_factory):
    subprocess.run(["make", "-s", "-C", CPP], check=True)
    out = str(tmp_path_factory.mktemp("dropin") / "test_dropin")
    subprocess.run(["g++", "-std=c++20", "-O2", "-Wall", "-Wextra", f"-I{CPP}", f"-I{CPP}/compat",
                    f"-I{ROOT}/include", "-o", out, os.path.join(ROOT, "tests", "cpp", "test_dropin.cpp"),
                    f"-L{CPP}", "-l:libdirktensor_dropin.so", f"-Wl,-rpath,{CPP}",
                    f"-L{ROOT}/dirktensor_b200", "-l:libdirktensor_b200.so", f"-Wl,-rpath,{ROOT}/dirktensor_b200"],
                   check=True)
    return out


def test_dropin_flash_attention_forward(cuda, dropin_bin, tmp_path):
    B, T, H = 2, 300, 4
    q, k, v = qkv(31, B, T, H)
    do = randn(32, q.shape)
    for n, a in (("q", q), ("k", k), ("v", v), ("do", do)):
        a.tofile(tmp_path / f"{n}.f32")
    subprocess.run([dropin_bin, "flash", str(tmp_path), str(B), str(T), str(H)], check=True)
    o = np.fromfile(tmp_path / "o.f32", np.float32).reshape(B, T, H, 128)
    m = np.fromfile(tmp_path / "m.f32", np.float32).reshape(B, T, H)
    ro, rm, rl = oracle.flash_fwd(q, k, v, SCALE, True)
    assert rel_l2(o, ro) < TOL_ATTN_REL_L2
    assert np.max(np.abs(m - rm)) < 5e-2
    # flash_attention_backward through the drop-in (on the drop-in's own forward outputs)
    l = np.fromfile(tmp_path / "l.f32", np.float32).reshape(B, T, H)
    ref = oracle.flash_bwd(do, o, m, l, q, k, v, SCALE, True)
    for n, r in zip(("dq", "dk", "dv"), ref):
        got = np.fromfile(tmp_path / f"{n}.f32", np.float32).reshape(B, T, H, 128)
        assert rel_l2(got, r) < TOL_BWD_REL_L2, n


def test_dropin_olmo_attention_block_usage(cuda, dropin_bin, tmp_path):
    ws = layer_weights(32)
    for n, w in zip(["q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm"], ws):
        np.save(tmp_path / f"model.layers.5.self_attn.{n}.weight.npy", w)
    B, T = 2, 96
    x = randn(33, (B, T, 2048))
    x.tofile(tmp_path / "x.f32")
    subprocess.run([dropin_bin, "layer", str(tmp_path), "5", str(B), str(T)], check=True)
    y = np.fromfile(tmp_path / "y.f32", np.float32).reshape(B, T, 2048)
    ref = oracle.attention_layer(x, *ws)
    assert rel_l2(y, ref) < TOL_LAYER_REL_L2
    # a missing layer surfaces as a C++ exception -> non-zero exit
    r = subprocess.run([dropin_bin, "layer", str(tmp_path), "6", str(B), str(T)], capture_output=True, text=True)
    assert r.returncode == 1 and "cannot open" in r.stderr


@pytest.mark.parametrize("world", [1, 2])
def test_dropin_olmo_attention_head_parallel(cuda, dropin_bin, tmp_path, world):
    """dirktensor_b200::set_tensor_parallel(comm): the same OlmoBlock-style owner,
    unchanged, holds only this rank's heads; every rank's forward returns the
    whole output.  One process per GPU (rank = GPU), NCCL id through a file."""
    import torch

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ws = layer_weights(34)
    for n, w in zip(["q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm"], ws):
        np.save(tmp_path / f"model.layers.3.self_attn.{n}.weight.npy", w)
    B, T = 2, 320
    x = randn(35, (B, T, 2048))
    x.tofile(tmp_path / "x.f32")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([dropin_bin, "layer_tp", str(tmp_path), "3", str(B), str(T), str(world), str(r)],
                              env=env) for r in range(world)]
    for p in procs:
        assert p.wait(timeout=300) == 0
    ref = oracle.attention_layer(x, *ws)
    for r in range(world):
        y = np.fromfile(tmp_path / f"y{r}.f32", np.float32).reshape(B, T, 2048)
        assert rel_l2(y, ref) < TOL_LAYER_REL_L2, r


def test_dropin_olmo_attention_training_calls(cuda, dropin_bin, tmp_path):
    """forward -> backward -> step -> forward, as OlmoBlock drives it (OlmoBlock.cpp:14,28,33)."""
    ws = layer_weights(34)
    for n, w in zip(["q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm"], ws):
        np.save(tmp_path / f"model.layers.2.self_attn.{n}.weight.npy", w)
    B, T = 1, 100
    x = randn(35, (B, T, 2048))
    dy = randn(36, (B, T, 2048))
    x.tofile(tmp_path / "x.f32")
    dy.tofile(tmp_path / "dy.f32")
    subprocess.run([dropin_bin, "train", str(tmp_path), "2", str(B), str(T)], check=True)
    dx = np.fromfile(tmp_path / "dx.f32", np.float32).reshape(B, T, 2048)
    y2 = np.fromfile(tmp_path / "y2.f32", np.float32).reshape(B, T, 2048)
    _, saved = oracle.attention_layer_train(x, *ws)
    rdx, g = oracle.attention_layer_backward(dy, saved, *ws)
    assert rel_l2(dx, rdx) < TOL_LAYER_BWD_REL_L2
    keys = ["q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm"]
    stepped = [w - np.float32(1e-3) * g[k] for w, k in zip(ws, keys)]
    assert rel_l2(y2, oracle.attention_layer(x, *stepped)) < TOL_LAYER_REL_L2


def test_dropin_olmo_model(cuda, dropin_bin, tmp_path):
    """OlmoModel(folder).forward(batch) -> logits, as test_olmo_model.cpp:24-45 calls it."""
    from test_model_gpu import KEYS, model_weights

    embed, layers, final_norm, lm_head = model_weights(9, 2, 512)
    np.save(tmp_path / "model.embed_tokens.weight.npy", embed)
    np.save(tmp_path / "model.norm.weight.npy", final_norm)
    np.save(tmp_path / "lm_head.weight.npy", lm_head)
    names = {"post_attention_norm": "post_attention_layernorm", "post_feedforward_norm": "post_feedforward_layernorm",
             "gate_proj": "mlp.gate_proj", "up_proj": "mlp.up_proj", "down_proj": "mlp.down_proj"}
    for i, lw in enumerate(layers):
        for k in KEYS:
            np.save(tmp_path / f"model.layers.{i}.{names.get(k, 'self_attn.' + k)}.weight.npy", lw[k])
    ids = np.random.default_rng(4).integers(0, 512, (2, 48)).astype(np.uint32)
    ids.tofile(tmp_path / "ids.u32")
    subprocess.run([dropin_bin, "model", str(tmp_path), "2", "2", "48"], check=True)
    got = np.fromfile(tmp_path / "logits.f32", np.float32).reshape(2, 48, 512)
    ref = oracle.model_forward(ids, embed, layers, final_norm, lm_head)
    assert rel_l2(got, ref) < 3e-2
