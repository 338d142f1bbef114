"""Data-parallel execution across the GPUs of one box.

The path shards by batch: images are independent and the integer pass is
batch-size invariant (the reference's own test_container.py:201-206), so
each rank runs a full replica on a contiguous slice of the batch with no
collective on the data path.  Two collectives exist, both small:

* calibration: every rank observes its shard of the calibration batches;
  the per-tensor (min, max) ranges are combined with one all-reduce
  (MIN of the lows, MAX of the highs) before ``finalize``, so all ranks
  derive identical qparams -- exactly the ranges a single process would see
  (min / max are order independent);
* output gather: the per-rank float32 outputs are gathered into the full
  batch.

Backend: ``torch.distributed`` -- NCCL over NVLink on GPUs, gloo on CPU
(tests).  One process per GPU.
"""

import os
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist


def init(backend=None, timeout_s=120):
    """Initializes the default process group from torchrun's environment."""
    if dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
    if backend == "nccl":
        local = int(os.environ.get("LOCAL_RANK", 0))
        torch.cuda.set_device(local)
        from quantanything_b200 import native

        native.get_library().set_device(local)
    dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s))
    return dist.get_rank(), dist.get_world_size()


def shard_bounds(total, rank, world):
    """Contiguous ``[lo, hi)`` slice of ``total`` items for ``rank``; shards
    differ in size by at most one."""
    base, extra = divmod(int(total), int(world))
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard(x, rank, world):
    lo, hi = shard_bounds(len(x), rank, world)
    return x[lo:hi]


def _device_for(group):
    backend = dist.get_backend(group)
    if backend == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def allreduce_ranges(ranges, group=None):
    """Combines ``{key: (lo, hi)}`` across ranks: MIN of lows, MAX of highs.

    Every rank must hold the same keys (same graph, every tensor observed);
    the packed vector is ordered by sorted key, so ranks agree without
    exchanging names.  Returns the combined dict on every rank.
    """
    keys = sorted(ranges)
    dev = _device_for(group)
    lo = torch.tensor([ranges[k][0] for k in keys], dtype=torch.float64, device=dev)
    neg_hi = torch.tensor([-ranges[k][1] for k in keys], dtype=torch.float64, device=dev)
    packed = torch.stack([lo, neg_hi])
    dist.all_reduce(packed, op=dist.ReduceOp.MIN, group=group)
    packed = packed.cpu().numpy()
    return {k: (float(packed[0, i]), float(-packed[1, i])) for i, k in enumerate(keys)}


def gather_outputs(y, total, group=None):
    """All-gathers per-rank output shards (float32 [n_r, C], contiguous
    shards in rank order) into the full [total, C] array on every rank.
    ``y`` may be a host array or a tensor; a tensor already on the group's
    device is gathered there and the result stays a device tensor (only
    host inputs come back as a NumPy array)."""
    world = dist.get_world_size(group)
    dev = _device_for(group)
    on_device = isinstance(y, torch.Tensor) and y.device == dev and dev.type == "cuda"
    t = y if on_device else torch.as_tensor(np.ascontiguousarray(
        y.cpu().numpy() if isinstance(y, torch.Tensor) else y)).to(dev)
    spans = [shard_bounds(total, r, world) for r in range(world)]
    rows = max(hi - lo for lo, hi in spans)
    # collectives move equal-sized buffers: pad every shard to the largest
    padded = torch.zeros((rows, *t.shape[1:]), dtype=t.dtype, device=dev)
    padded[: t.shape[0]] = t
    buf = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(buf, padded, group=group)
    full = torch.cat([b[: hi - lo] for b, (lo, hi) in zip(buf, spans)])
    return full if on_device else full.cpu().numpy()


def gather_outputs_device(y, out, group=None):
    """All-gathers equal-sized per-rank output shards that are already on the
    group's device: ``y`` [n, C] on every rank -> ``out`` [world * n, C]
    (rank order), one ``all_gather_into_tensor`` enqueued on the current
    stream -- no host round trip.  Returns ``out``."""
    world = dist.get_world_size(group)
    if out.shape[0] != world * y.shape[0] or out.shape[1:] != y.shape[1:]:
        raise ValueError(f"gather buffer {tuple(out.shape)} does not hold {world} shards of "
                         f"{tuple(y.shape)}")
    dist.all_gather_into_tensor(out, y.contiguous(), group=group)
    return out


def calibrate_sharded(container, batches, group=None):
    """Each rank calibrates on its shard of ``batches`` (a list of arrays,
    split by index), ranges are all-reduced, then every rank finalizes."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    mine = [b for i, b in enumerate(batches) if i % world == rank]
    if not mine:
        raise ValueError("fewer calibration batches than ranks")
    container.calibrate(mine, reduce_ranges=lambda r: allreduce_ranges(r, group))
    return container
