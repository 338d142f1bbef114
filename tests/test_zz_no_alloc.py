"""The allocation-free GEMM entry point matches the regular one (B200).

qa_gemm_i16_i32_noalloc_dev serves callers that cannot allocate GPU memory
while they run (a service that reserved its device memory up front, a host
runtime that hands over only its own input and output buffers); it packs
operands into a fixed library-owned device array instead of buffers grown
with cudaMalloc.  Called through the C ABI on device buffers, its results
must equal the existing qa_gemm_i16_i32 entry point's bit for bit, on
consecutive calls (the scratch array is shared and keeps the previous
call's contents), its status word must read clean afterwards, and calls
after the first must leave the device's free memory unchanged.  This file
is collected last so a failure here never hides the other tests' results.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _entry(lib):
    fn = lib.raw.qa_gemm_i16_i32_noalloc_dev
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 3 + [ctypes.c_void_p]
    size = lib.raw.qa_noalloc_scratch_bytes
    size.restype, size.argtypes = ctypes.c_int64, []
    status = lib.raw.qa_noalloc_status_dev
    status.restype, status.argtypes = ctypes.c_int, [ctypes.c_void_p]
    return fn, size()


def _status(lib, stream):
    rc = lib.raw.qa_noalloc_status_dev(stream)
    assert rc == 0, lib.raw.qa_last_error()


def test_noalloc_gemm_matches_regular_entry_point_on_consecutive_calls(gpu_lib):
    import torch

    fn, scratch = _entry(gpu_lib)
    assert scratch == 16 << 20
    stream = torch.cuda.current_stream().cuda_stream
    for (m, k, n), seed in [((300, 1000, 200), 1), ((77, 64, 513), 2), ((5, 3, 7), 3)]:
        rng = np.random.default_rng(seed)
        a = rng.integers(-(2**15), 2**15, (m, k)).astype(np.int16)
        b = rng.integers(-(2**15), 2**15, (k, n)).astype(np.int16)
        expect = gpu_lib.gemm_int(a, b, False)  # regular host-pointer entry point
        da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        dc = torch.full((m, n), -1, dtype=torch.int32, device="cuda")
        rc = fn(da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, n, k, stream)
        assert rc == 0, gpu_lib.raw.qa_last_error()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(dc.cpu().numpy(), expect)
        _status(gpu_lib, stream)


def test_noalloc_gemm_leaves_free_memory_unchanged(gpu_lib):
    import torch

    fn, _ = _entry(gpu_lib)
    stream = torch.cuda.current_stream().cuda_stream
    m, k, n = 256, 768, 512
    rng = np.random.default_rng(5)
    a = rng.integers(-(2**15), 2**15, (m, k)).astype(np.int16)
    b = rng.integers(-(2**15), 2**15, (k, n)).astype(np.int16)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    dc = torch.empty((m, n), dtype=torch.int32, device="cuda")
    assert fn(da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, n, k, stream) == 0
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        assert fn(da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, n, k, stream) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    _status(gpu_lib, stream)
    np.testing.assert_array_equal(dc.cpu().numpy(), gpu_lib.gemm_int(a, b, False))


def test_noalloc_gemm_rejects_oversized_request(gpu_lib):
    import torch

    fn, scratch = _entry(gpu_lib)
    m, k, n = 8192, 2048, 64  # ~32 MiB of packed planes
    da = torch.zeros((1,), dtype=torch.int16, device="cuda")
    rc = fn(da.data_ptr(), da.data_ptr(), da.data_ptr(), m, n, k,
            torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    msg = gpu_lib.raw.qa_last_error().decode()
    assert "scratch" in msg and str(scratch) in msg
    gpu_lib.raw.qa_clear_error()
