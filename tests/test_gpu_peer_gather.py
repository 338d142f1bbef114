"""Output dequantize fused with the multi-GPU gather (B200, NVLink peer memory).

Each rank runs qa_dequantize_gather_peers_dev once per step: its int32
output rows are dequantized as the reference does (qa_kernels.cpp:378-386,
x = float((double)(q - zp) * scale)) and stored into every rank's buffer.
Two ranks on two GPUs run several epochs with fresh outputs each step (both
slots reused twice); every rank's gathered batch must equal the reference
dequantize of all ranks' rows, bit for bit.  The single-GPU test makes the
kernel's bounded wait run out: a second "rank" whose buffer exists but
whose process never runs, so its flag is never raised.
"""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
K_DEVICE_TIMEOUT = 3
ROWS, COLS, EPOCHS = 48, 1000, 5
SCALE, ZP = 0.0039215689, -7


def _rank_output(rank, epoch):
    rng = np.random.default_rng(1000 * epoch + rank)
    return rng.integers(-128, 128, (ROWS, COLS)).astype(np.int32)


def _reference_dequantize(q):
    return ((q.astype(np.int64) - ZP).astype(np.float64) * SCALE).astype(np.float32)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, errors):
    from datetime import timedelta

    import torch.distributed as dist

    from quantanything_b200 import distributed, native

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        lib = native.get_library()
        lib.set_device(rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        pg = distributed.PeerGather(ROWS, COLS, budget_s=10.0)
        for epoch in range(1, EPOCHS + 1):
            q = torch.from_numpy(_rank_output(rank, epoch)).cuda()
            got = pg(q, SCALE, ZP).cpu().numpy()  # the copy follows the kernel on the stream
            want = np.concatenate([_reference_dequantize(_rank_output(r, epoch))
                                   for r in range(world)])
            if not np.array_equal(got.view(np.uint32), want.view(np.uint32)):
                raise AssertionError(f"rank {rank} epoch {epoch}: gathered rows differ")
        rc = lib.raw.qa_device_status_dev(
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        if rc != 0:
            raise AssertionError(f"rank {rank}: device status {rc}")
        pg.close()
        dist.destroy_process_group()
    except BaseException as e:  # reported by the parent
        errors.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def test_two_ranks_gather_dequantized_rows_over_peer_memory():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    errors = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, errors)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not alive, "a rank did not finish"
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs)


def test_missing_rank_makes_the_gather_wait_run_out(gpu_lib):
    """world = 2 in one process: rank 1's buffer is allocated here, but no
    rank 1 ever runs, so the flag this rank waits for is never raised."""
    from quantanything_b200.distributed import IPC_HANDLE_BYTES, peer_api
    from quantanything_b200.resident import device_api

    raw = peer_api(gpu_lib)
    device_api(gpu_lib)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert raw.qa_device_status_dev(st) == 0
    header = raw.qa_peer_buffer_header_bytes()
    bufs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        h = (ctypes.c_uint8 * IPC_HANDLE_BYTES)()
        assert raw.qa_peer_buffer_create(header + 2 * 4 * 2 * ROWS * COLS, ctypes.byref(p), h) == 0
        bufs.append(p.value)
    bases = (ctypes.c_void_p * 2)(*bufs)
    q = torch.from_numpy(_rank_output(0, 1)).cuda()
    budget_ns = 20_000_000  # 20 ms
    assert raw.qa_dequantize_gather_peers_dev(q.data_ptr(), COLS, ZP, SCALE, ROWS, COLS, bases,
                                              2, 0, 1, budget_ns, st) == 0
    assert raw.qa_device_status_dev(st) == K_DEVICE_TIMEOUT
    gpu_lib.raw.qa_clear_error()
    assert raw.qa_device_status_dev(st) == 0
    # this rank's own rows still landed in slot 1 of its buffer
    mine = torch.empty((ROWS, COLS), dtype=torch.float32)
    view = torch.as_tensor(_view(bufs[0] + header + 4 * 2 * ROWS * COLS), device="cuda")
    mine.copy_(view[:ROWS])
    np.testing.assert_array_equal(mine.numpy(), _reference_dequantize(_rank_output(0, 1)))
    torch.cuda.synchronize()
    for p in bufs:
        assert raw.qa_peer_buffer_destroy(p) == 0


def _view(ptr):
    from quantanything_b200.distributed import _DeviceView

    return _DeviceView(ptr, (2 * ROWS, COLS))


def test_gather_rejects_bad_arguments(gpu_lib):
    from quantanything_b200.distributed import peer_api

    raw = peer_api(gpu_lib)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    bases = (ctypes.c_void_p * 1)(None)
    q = torch.zeros((2, 4), dtype=torch.int32, device="cuda")
    assert raw.qa_dequantize_gather_peers_dev(q.data_ptr(), 4, 0, 1.0, 2, 4, bases, 1, 0, 1,
                                              1000, st) != 0  # unmapped buffer
    gpu_lib.raw.qa_clear_error()
    assert raw.qa_dequantize_gather_peers_dev(q.data_ptr(), 4, 0, 1.0, 2, 4, bases, 9, 0, 1,
                                              1000, st) != 0  # world above 8
    gpu_lib.raw.qa_clear_error()
