"""GPU test of dt_flash_fwd_noalloc, the flash-attention entry point for callers
that cannot allocate device memory (an engine that owns its HBM budget through
its own pool, a plugin barred from allocating, a loop that cannot afford
cudaMalloc's synchronisation).  Its scratch is a fixed array inside the library,
shared by every call.  It is called here through the C ABI twice in a row, on
different shapes.  Each result must be bit-identical to the workspace entry
point dt_flash_fwd on the same inputs (both round K and V to nearest-even bf16
and round Q inside the attention kernel), and within the attention tolerances
of the oracle.  Kept in its own file, collected last."""
import ctypes

import numpy as np
import pytest

import oracle
from common import SCALE, TOL_ATTN_MAX_ABS, TOL_ATTN_REL_L2, TOL_L_REL, TOL_M_ABS, max_abs, qkv, rel_l2

pytestmark = pytest.mark.gpu


def _run(fn_name, cuda, q, k, v, causal=True):
    import torch

    from dirktensor_b200._lib import check, lib

    Q, K, V = (torch.from_numpy(a).to(cuda) for a in (q, k, v))
    B, T, H, D = q.shape
    o = torch.empty_like(Q)
    m = torch.empty((B, T, H), device=cuda)
    l = torch.empty((B, T, H), device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    L = lib()
    if fn_name == "noalloc":
        st = L.dt_flash_fwd_noalloc(Q.data_ptr(), K.data_ptr(), V.data_ptr(), o.data_ptr(), m.data_ptr(),
                                    l.data_ptr(), B, T, H, D, SCALE, int(causal), stream)
    else:
        ws = torch.empty(L.dt_flash_fwd_workspace_bytes(B, T, H, D), dtype=torch.uint8, device=cuda)
        st = L.dt_flash_fwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), o.data_ptr(), m.data_ptr(), l.data_ptr(),
                            B, T, H, D, SCALE, int(causal), ws.data_ptr(), ws.numel(), stream)
    check(st)
    check(L.dt_check_device_error())
    return o.cpu().numpy(), m.cpu().numpy(), l.cpu().numpy()


def test_noalloc_matches_workspace_entry_point_twice(cuda):
    # the second call reuses the scratch the first one left behind
    cases = [((1, 2048, 16), True), ((2, 300, 3), False)]
    for (B, T, H), causal in cases:
        q, k, v = qkv(900 + T, B, T, H)
        o, m, l = _run("noalloc", cuda, q, k, v, causal)
        ro, rm, rl = _run("workspace", cuda, q, k, v, causal)
        assert np.array_equal(o, ro) and np.array_equal(m, rm) and np.array_equal(l, rl)
        eo, em, el = oracle.flash_fwd(q, k, v, SCALE, causal)
        assert rel_l2(o, eo) < TOL_ATTN_REL_L2
        assert max_abs(o, eo) < TOL_ATTN_MAX_ABS
        assert max_abs(m, em) < TOL_M_ABS
        assert np.max(np.abs(l - el) / np.abs(el)) < TOL_L_REL


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    from dirktensor_b200._lib import lib

    L = lib()
    # 1 x 3073 x 16 x 128 elements exceed the 6,291,456-element limit; rejected before any launch
    st = L.dt_flash_fwd_noalloc(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16),
                                None, None, 1, 3073, 16, 128, SCALE, 1, None)
    assert st == 1
    assert b"exceeds the fixed scratch" in L.dt_last_error()
