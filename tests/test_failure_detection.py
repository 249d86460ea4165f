"""Failure detection on the GPU without a GPU fault.

Every mbarrier wait of the tensor-core GEMM is bounded.  A test-only knob
(ima_set_gemm_wait_test) makes the MMA thread wait on a barrier that nothing arrives on;
the wait runs out, the kernel records IMA_ERR_TIMEOUT in the device status word, drains
the copies and tensor-core work it has in flight and returns.  The context stays usable:
the next launch computes the exact product.  Nothing here traps, faults or hangs.
"""

from __future__ import annotations

import pytest
import torch

import oracle
from int_model_approximation_b200 import _native as nat
from int_model_approximation_b200 import students

pytestmark = pytest.mark.gpu

WHERE_GEMM_MMA = 3


def test_gemm_wait_that_runs_out_is_reported_and_the_next_call_is_exact(cuda_device):
    g = torch.Generator().manual_seed(3)
    a = torch.randint(-100, 100, (200, 96), generator=g, dtype=torch.int32)
    b = torch.randint(-100, 100, (96, 170), generator=g, dtype=torch.int32)
    a_d, b_d = a.to(cuda_device), b.to(cuda_device)
    nat.device_status(cuda_device.index or 0, clear=True)
    nat.call("ima_set_gemm_wait_test", 50_000)   # 50 microseconds
    try:
        students._int32_raw_matmul(a_d, b_d)       # returns: the launch gives up and drains
        code, where, detail = nat.device_status(cuda_device.index or 0, clear=True)
    finally:
        nat.call("ima_set_gemm_wait_test", 0)
    assert code == nat.IMA_ERR_TIMEOUT
    assert (where, detail) == (WHERE_GEMM_MMA, -2)
    c = students._int32_raw_matmul(a_d, b_d)
    assert torch.equal(c.cpu(), oracle.int_gemm(a, b))
    assert nat.device_status(cuda_device.index or 0, clear=True) == (0, 0, 0)


def test_gemm_wait_test_knob_rejects_out_of_range_values():
    lib = nat.lib()
    assert lib.ima_set_gemm_wait_test(-1) == nat.IMA_ERR_INVALID_ARGUMENT
    assert lib.ima_set_gemm_wait_test(3_000_000_000) == nat.IMA_ERR_INVALID_ARGUMENT
    assert lib.ima_set_gemm_wait_test(0) == nat.IMA_OK
