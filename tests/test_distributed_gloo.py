"""Multi-process (world size 2, gloo on CPU) tests of the data-parallel path.

Sharded calibration with the MIN/MAX all-reduce must give exactly the
qparams of one process calibrating on all batches, and the output gather
must reassemble the batch in order.  The kernel library is the C oracle
(CPU), so no GPU is involved.
"""
import json
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from tests.conftest import ORACLE_LIB, _ensure_oracle


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    import torch.distributed as dist

    from quantanything_b200 import distributed, networks
    from quantanything_b200.container import QuantContainer
    from quantanything_b200.native import KernelLibrary

    distributed.init("gloo", timeout_s=60)
    lib = KernelLibrary(ORACLE_LIB)
    qc = QuantContainer(networks.yolo_mini(width=16), "int8", lib=lib)
    batches = [networks.images(3, 32, seed=50 + i) for i in range(4)]
    distributed.calibrate_sharded(qc, batches)
    qc.save(os.path.join(outdir, f"q{rank}.json"))
    # the device calibration's path: per-rank range tables reduced with one
    # all-reduce of the packed (lo, -hi) table (CPU tensors and NumPy
    # stand-ins of the kernels here)
    from tests.fake_float_kernels import FakeLibrary

    qd = QuantContainer(networks.yolo_mini(width=16), "int8", lib=lib)
    distributed.calibrate_sharded(qd, batches, device="cpu", lib=FakeLibrary(lib))
    qd.save(os.path.join(outdir, f"d{rank}.json"))
    # each rank runs its shard of a 5-image batch; gather reassembles it
    x = networks.images(5, 32, seed=9)
    y = qc.run_graph(distributed.shard(x, rank, world), "integer")
    full = distributed.gather_outputs(y, len(x))
    np.save(os.path.join(outdir, f"y{rank}.npy"), full)
    # equal shards already in tensors: one all_gather_into_tensor, rank order
    import torch

    shard_t = torch.as_tensor(np.asarray(y, np.float32))[:2]
    gathered = torch.empty((world * 2, shard_t.shape[1]), dtype=torch.float32)
    distributed.gather_outputs_device(shard_t, gathered)
    np.save(os.path.join(outdir, f"g{rank}.npy"), gathered.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_calibration_and_gather(tmp_path):
    _ensure_oracle()
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    from quantanything_b200 import networks
    from quantanything_b200.container import QuantContainer
    from quantanything_b200.native import KernelLibrary

    lib = KernelLibrary(ORACLE_LIB)
    single = QuantContainer(networks.yolo_mini(width=16), "int8", lib=lib)
    single.calibrate([networks.images(3, 32, seed=50 + i) for i in range(4)])
    single.save(tmp_path / "single.json")
    ref = json.loads((tmp_path / "single.json").read_text())
    for r in range(world):
        assert json.loads((tmp_path / f"q{r}.json").read_text()) == ref
    # device-path tables: identical on both ranks, and the single process's
    # qparams up to the stand-in GEMM's float32 summation order
    d0 = json.loads((tmp_path / "d0.json").read_text())
    assert json.loads((tmp_path / "d1.json").read_text()) == d0
    for name, want in ref["qparams"].items():
        got = d0["qparams"][name]
        assert (got["qmin"], got["qmax"]) == (want["qmin"], want["qmax"]), name
        assert abs(got["zp"] - want["zp"]) <= 1, name
        assert abs(got["scale"] - want["scale"]) <= 1e-5 * abs(want["scale"]), name
    expect = single.run_graph(networks.images(5, 32, seed=9), "integer")
    for r in range(world):
        np.testing.assert_array_equal(np.load(tmp_path / f"y{r}.npy"), expect)
    # ranks hold images [0, 3) and [3, 5): their first two rows, in rank order
    for r in range(world):
        np.testing.assert_array_equal(np.load(tmp_path / f"g{r}.npy"), expect[[0, 1, 3, 4]])


def test_shard_bounds_cover_batch():
    from quantanything_b200.distributed import shard_bounds

    for total in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1


def test_rank_failure_is_reported_not_hung(tmp_path):
    """A rank that raises before the collective ends the job with an error
    (the survivor's collective times out) instead of hanging."""
    _ensure_oracle()
    port = _free_port()
    with pytest.raises(Exception):
        mp.start_processes(_failing_worker, args=(2, port), nprocs=2, start_method="spawn",
                           join=True)


def _failing_worker(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    import torch

    from quantanything_b200 import distributed

    distributed.init("gloo", timeout_s=10)
    if rank == 1:
        raise RuntimeError("injected host-side failure on rank 1")
    distributed.allreduce_ranges({"t": (0.0, 1.0)})
    torch.distributed.destroy_process_group()
