"""GPU test of failure detection without a GPU fault: a kernel waits on a barrier
that nothing arrives on; the bounded wait expires after its budget, the kernel
records the site and returns, the host sees DT_ERR_DEVICE_TIMEOUT through the
C ABI, and the same context then runs ordinary work correctly."""
import numpy as np
import pytest

import oracle
from common import SCALE, qkv, rel_l2

pytestmark = pytest.mark.gpu


def test_expired_wait_is_reported_and_context_survives(cuda):
    import torch

    import dirktensor_b200 as dt
    from dirktensor_b200._lib import lib

    assert lib().dt_selftest_expired_wait() == 0, lib().dt_last_error()
    assert lib().dt_check_device_error() == 0  # the word was cleared
    q, k, v = qkv(3, 1, 200, 2)
    r = dt.flash_attention_forward(*(torch.from_numpy(a).to(cuda) for a in (q, k, v)), SCALE, True)
    dt.check_device_error()
    ro, _, _ = oracle.flash_fwd(q, k, v, SCALE, True)
    assert rel_l2(r.output.cpu().numpy(), ro) < 1e-2
