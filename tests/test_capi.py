"""CPU tests of the C ABI library: it loads, exports every symbol the header
declares, validates arguments before touching a device, and its host-side RoPE
tables equal the oracle's (compute_rope_buffers, OlmoAttention.cpp:18-36)."""
import ctypes
import os
import re

import numpy as np

import oracle
from dirktensor_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dirktensor_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dt_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(_lib.LIB_PATH)
    syms = declared_symbols()
    assert len(syms) >= 15
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, f"missing exports: {missing}"
    # the Python binding covers the same set
    assert set(syms) == set(_lib.SIGNATURES), set(syms) ^ set(_lib.SIGNATURES)


def test_version_and_error_string():
    L = _lib.lib()
    assert L.dt_version() >= 100
    assert isinstance(L.dt_last_error(), bytes)


def test_argument_validation_without_device():
    L = _lib.lib()
    # head_dim 64 is rejected before any CUDA call
    st = L.dt_flash_fwd(None, None, None, None, None, None, 1, 16, 2, 64, 0.1, 1, None, 0, None)
    assert st == 4 and b"head_dim" in L.dt_last_error()
    # K not a multiple of 8
    st = L.dt_gemm_bf16_tn(None, None, None, 0, 16, 16, 12, 16, None)
    assert st == 1 and b"K" in L.dt_last_error()
    # cast count not a multiple of 4
    st = L.dt_cast_f32_bf16(None, None, 6, None)
    assert st == 1
    # empty problems are a no-op success
    assert L.dt_flash_fwd(None, None, None, None, None, None, 0, 16, 2, 128, 0.1, 1, None, 0, None) == 0
    assert L.dt_gemm_bf16_tn(None, None, None, 0, 0, 16, 64, 16, None) == 0
    # T beyond the RoPE table (model_config.h:4) is rejected
    st = L.dt_qk_norm_rope(None, None, None, 6144, None, None, None, None, None, 1, 9000, 1e-6, 5e5, None)
    assert st == 1 and b"max_seq_len" in L.dt_last_error()
    assert L.dt_attn_forward(None, None, 1, 1, None, None, None) == 1
    h = ctypes.c_void_p()
    st = L.dt_attn_create_from_npy(b"/nonexistent-folder", 0, 0, ctypes.byref(h))
    assert st == 6 and b"cannot open" in L.dt_last_error()


def test_qf32_entry_points_validate_before_device():
    L = _lib.lib()
    fake = 0x10000  # 16-byte aligned, never dereferenced: every case fails validation first
    # head_dim 64
    st = L.dt_flash_fwd_qf32(None, None, None, None, 0, 128, None, None, None, 1, 16, 2, 64, 0.1, 1, None)
    assert st == 4 and b"head_dim" in L.dt_last_error()
    # null q
    st = L.dt_flash_fwd_qf32(None, fake, fake, fake, 0, 256, None, None, None, 1, 16, 2, 128, 0.1, 1, None)
    assert st == 1 and b"null" in L.dt_last_error()
    # misaligned q
    st = L.dt_flash_fwd_qf32(fake + 4, fake, fake, fake, 0, 256, None, None, None, 1, 16, 2, 128, 0.1, 1, None)
    assert st == 1 and b"aligned" in L.dt_last_error()
    # output row stride below H*D
    st = L.dt_flash_fwd_qf32(fake, fake, fake, fake, 0, 128, None, None, None, 1, 16, 2, 128, 0.1, 1, None)
    assert st == 1 and b"o_row_stride" in L.dt_last_error()
    # empty problem: no-op success
    assert L.dt_flash_fwd_qf32(None, None, None, None, 0, 256, None, None, None, 0, 16, 2, 128, 0.1, 1, None) == 0
    bufs = (ctypes.c_void_p * 2)(fake, fake)
    # rank out of range, token split that does not cover B*T
    st = L.dt_flash_fwd_qf32_exchange(fake, fake, fake, bufs, 2, 2, 8, None, None, 1, 16, 2, 128, 0.1, 1, None)
    assert st == 1 and b"rank" in L.dt_last_error()
    st = L.dt_flash_fwd_qf32_exchange(fake, fake, fake, bufs, 2, 0, 7, None, None, 1, 16, 2, 128, 0.1, 1, None)
    assert st == 1 and b"tokens_per_rank" in L.dt_last_error()


def test_qf32_python_wrapper_rejects_host_tensors():
    import pytest
    import torch

    import dirktensor_b200 as dt

    q = torch.zeros((1, 16, 2, 128))
    kb = torch.zeros((1, 16, 2, 128), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="q must be"):
        dt.flash_attention_forward_qf32(q, kb, kb, 0.1)


def test_workspace_size():
    L = _lib.lib()
    n = 2 * 300 * 16 * 128
    assert L.dt_flash_fwd_workspace_bytes(2, 300, 16, 128) >= 3 * n * 2
    assert L.dt_flash_fwd_workspace_bytes(0, 300, 16, 128) == 0


def test_rope_tables_equal_oracle():
    import dirktensor_b200 as dt

    s, c = dt.rope_tables(8192, 128, 500000.0)
    os_, oc = oracle.rope_tables(8192, 128, 500000.0)
    assert np.array_equal(s, os_) and np.array_equal(c, oc)


def test_head_parallel_entry_points_validate_before_any_device_work():
    """The communicator, sharded-layer, barrier and sharded-prologue entry points
    reject bad arguments (world size, ranks, sizes, null handles) before they
    touch a device or NCCL."""
    L = _lib.lib()
    uid = (ctypes.c_uint8 * 128)()
    comm = ctypes.c_void_p()
    assert L.dt_comm_create(uid, 9, 0, 0, 1000, ctypes.byref(comm)) == 1      # world > 8
    assert L.dt_comm_create(uid, 2, 2, 0, 1000, ctypes.byref(comm)) == 1      # rank out of range
    assert L.dt_comm_create(uid, 2, 0, 0, 0, ctypes.byref(comm)) == 1         # no timeout
    assert L.dt_comm_destroy(None) == 0 and L.dt_comm_abort(None) == 0
    attn = ctypes.c_void_p()
    w = _lib.dt_attn_weights()
    assert L.dt_attn_create_sharded(ctypes.byref(w), None, 0, ctypes.byref(attn)) == 1
    assert L.dt_attn_forward_sharded(None, None, 1, 512, None, 0, None, None) == 1
    assert L.dt_attn_forward_sharded_host(None, None, 1, 512, None, 0, None) == 1
    flags = (ctypes.c_void_p * 2)(16, 16)
    assert L.dt_exchange_barrier(flags, 9, 0, 1, None) == 1                   # ranks > 8
    assert L.dt_exchange_barrier(flags, 2, 0, 0, None) == 1                   # epoch 0
    assert L.dt_exchange_barrier((ctypes.c_void_p * 2)(16, None), 2, 0, 1, None) == 1
    assert b"flag buffer" in L.dt_last_error()
    assert L.dt_qk_sumsq(None, None, 2048, 6, 4, None, None) == 1            # width % 4
    assert L.dt_qk_sumsq(None, None, 2048, 256, 0, None, None) == 0          # empty: no-op
    st = L.dt_qk_norm_rope_shard(None, None, None, 768, None, None, None, 3, None, None, None, 1, 4, 1e-6, 5e5, None)
    assert st == 1 and b"heads" in L.dt_last_error()
    assert L.dt_cast2_f32_bf16(None, None, None, None, 6, None) == 1
    assert L.dt_cast2_f32_bf16(None, None, None, None, 0, None) == 0


def test_gemm_backward_and_noalloc_validate_before_device():
    """The general and planar GEMM forms, the attention backward and the no-alloc
    forward reject bad shapes, strides, alignments and sizes before any CUDA call."""
    L = _lib.lib()
    fake = 1 << 20  # 16-byte aligned, never dereferenced
    # general form: bad c_mode, K not a multiple of 8 with a K-major operand, MN-major M % 8
    assert L.dt_gemm_bf16(fake, 0, fake, 0, fake, 3, 16, 16, 64, 16, None) == 1
    assert L.dt_gemm_bf16(fake, 0, fake, 0, fake, 0, 16, 16, 12, 16, None) == 1
    assert L.dt_gemm_bf16(fake, 1, fake, 1, fake, 0, 12, 16, 64, 16, None) == 1
    # ldc shorter than N, or leaving fp32 rows unaligned
    assert L.dt_gemm_bf16_tn(fake, fake, fake, 0, 16, 16, 64, 8, None) == 1
    assert L.dt_gemm_bf16_tn(fake, fake, fake, 0, 16, 16, 64, 18, None) == 1
    # unaligned operand
    assert L.dt_gemm_bf16_tn(fake + 4, fake, fake, 0, 16, 16, 64, 16, None) == 1
    # planar A: K must split into planes of a multiple of 64
    st = L.dt_gemm_bf16_tn_planar(fake, 3, fake, fake, 0, 16, 16, 2048, 16, None)
    assert st == 1 and b"planes" in L.dt_last_error()
    assert L.dt_gemm_bf16_tn_planar(fake, 4, fake, fake, 0, 16, 16, 96, 16, None) == 1
    # attention backward: head_dim, then a workspace too small for the shape
    st = L.dt_flash_bwd(*([None] * 10), 1, 16, 2, 64, 0.1, 1, None, 0, None)
    assert st == 4 and b"head_dim" in L.dt_last_error()
    ptrs = [fake] * 10
    st = L.dt_flash_bwd(*ptrs, 1, 16, 2, 128, 0.1, 1, fake, 64, None)
    assert st == 1 and b"workspace" in L.dt_last_error()
    assert L.dt_flash_bwd(*([None] * 10), 0, 16, 2, 128, 0.1, 1, None, 0, None) == 0  # empty: no-op
    # no-alloc forward: beyond its fixed scratch
    st = L.dt_flash_fwd_noalloc(fake, fake, fake, fake, None, None, 2, 4096, 16, 128, 0.1, 1, None)
    assert st == 1 and b"fixed scratch" in L.dt_last_error()
