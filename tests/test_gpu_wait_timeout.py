"""The bounded-wait error channel of the tensor-core kernels (B200).

Every mbarrier wait in the library is bounded; a wait that runs out records
a timeout in the device status word and the kernel returns instead of
hanging.  qa_wait_probe_dev runs that same bounded wait on an mbarrier
nothing arrives on (a short budget, no copy in flight): the next
qa_device_status_dev must report kDeviceTimeout, clear the word, and the
context must stay usable -- a released wait then reports nothing and a
resident kernel still computes the oracle's result.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
K_DEVICE_TIMEOUT = 3
BUDGET = 1 << 21  # SM cycles: about a millisecond


def test_bounded_wait_that_runs_out_is_reported(gpu_lib, oracle):
    from quantanything_b200.resident import device_api

    raw = device_api(gpu_lib)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert raw.qa_device_status_dev(st) == 0
    assert raw.qa_wait_probe_dev(BUDGET, 0, st) == 0  # nothing arrives
    assert raw.qa_device_status_dev(st) == K_DEVICE_TIMEOUT
    assert b"bounded wait" in raw.qa_last_error()
    gpu_lib.raw.qa_clear_error()
    assert raw.qa_device_status_dev(st) == 0  # the word was cleared
    assert raw.qa_wait_probe_dev(BUDGET, 1, st) == 0  # released: no timeout
    assert raw.qa_device_status_dev(st) == 0
    # the context is intact: a kernel afterwards matches the oracle
    rng = np.random.default_rng(4)
    a = rng.integers(-128, 128, (40, 64)).astype(np.int64)
    b = rng.integers(-127, 128, (64, 24)).astype(np.int64)
    np.testing.assert_array_equal(gpu_lib.gemm_int(a, b, False), oracle.gemm_int(a, b, False))


def test_wait_probe_rejects_unbounded_budget(gpu_lib):
    from quantanything_b200.resident import device_api

    raw = device_api(gpu_lib)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert raw.qa_wait_probe_dev((1 << 32) + 1, 0, st) != 0
    gpu_lib.raw.qa_clear_error()
