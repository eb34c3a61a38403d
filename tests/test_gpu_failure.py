"""Failure detection without a GPU fault: every wait inside the step kernels
is bounded. Here a wait on a flag that nothing raises expires, records
AOAKV_DEV_ERR_TIMEOUT in the device error word and returns, and the context
keeps working (no trap, no fault, no hang)."""
import time

import numpy as np
import pytest
import torch

from aoa_kv_b200 import _lib
from gpu_util import stream

pytestmark = pytest.mark.gpu

DEV_ERR_TIMEOUT = 2


def test_wait_on_unraised_flag_expires_and_reports(cuda):
    _lib.device_error()  # start clean
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.perf_counter()
    _lib.call("aoakv_debug_wait_flag", flag.data_ptr(), 1, 2000, stream())  # 2 ms limit
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert _lib.device_error() == DEV_ERR_TIMEOUT
    # the context is intact: a raised flag passes, and ordinary work runs
    flag.fill_(3)
    _lib.call("aoakv_debug_wait_flag", flag.data_ptr(), 3, 2000, stream())
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum().item()) == float(np.arange(1024).sum())
    assert _lib.device_error() == 0


def test_debug_wait_rejects_bad_limit(cuda):
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(Exception, match="limit_us"):
        _lib.call("aoakv_debug_wait_flag", flag.data_ptr(), 1, 0, stream())
