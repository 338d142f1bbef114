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
* output gather: the per-rank outputs are gathered into the full batch --
  on GPUs by ``PeerGather``, one kernel per rank that dequantizes the
  rank's int32 output rows and stores them into every rank's buffer over
  NVLink peer memory (no NCCL on that path); ``gather_outputs_device``
  (NCCL ``all_gather_into_tensor``) and ``gather_outputs`` (any backend,
  host or device tensors) remain for float32 shards.

Backend: ``torch.distributed`` -- NCCL over NVLink on GPUs, gloo on CPU
(tests).  One process per GPU.
"""

import ctypes
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


class _DeviceView:
    """A device pointer presented through ``__cuda_array_interface__`` so
    that torch can wrap it without a copy."""

    def __init__(self, ptr, shape, typestr="<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "strides": None,
                                         "version": 3}


_PEER_SIGNATURES = {
    "qa_peer_buffer_header_bytes": (ctypes.c_int64, []),
    "qa_peer_buffer_create": (ctypes.c_int, [ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p),
                                             ctypes.c_void_p]),
    "qa_peer_buffer_open": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "qa_peer_buffer_close": (ctypes.c_int, [ctypes.c_void_p]),
    "qa_peer_buffer_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "qa_dequantize_gather_peers_dev": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_double, ctypes.c_int64,
        ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32, ctypes.c_int32,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]),
}
IPC_HANDLE_BYTES = 64  # sizeof(cudaIpcMemHandle_t)


def peer_api(lib):
    """Declares the peer-buffer entry points on a loaded KernelLibrary."""
    raw = lib.raw
    if not getattr(raw, "_qa_peer_declared", False):
        for name, (res, args) in _PEER_SIGNATURES.items():
            fn = getattr(raw, name)
            fn.restype, fn.argtypes = res, args
        raw._qa_peer_declared = True
    return raw


class PeerGather:
    """The graph output's dequantize fused with the all-gather of the
    per-rank shards (quant_container.py:186-193 dequantizes each output;
    the batch shards are then collected in rank order).

    Each rank owns one device buffer, mapped into every other rank's
    process through CUDA IPC.  ``__call__(q, scale, zp)`` launches ONE
    kernel on the current stream (qa_dequantize_gather_peers_dev): it reads
    this rank's int32 output rows, dequantizes them and stores the float32
    rows into every rank's buffer over NVLink peer memory, then raises the
    rank's flag in each buffer and waits (bounded) for the other ranks'
    flags.  No NCCL call is made on this path.  The returned [world * rows,
    cols] float32 tensor (rank order) is valid once the stream reaches the
    end of the kernel and until the next call's kernel starts on this
    stream: that launch tells the other ranks that this rank is done with
    the slot, which they reuse one call later (two alternating slots).  A
    rank that stops calling makes the others' waits
    run out after ``budget_s`` with the device status set to a timeout.

    Every rank must construct it (collective) and call it the same number
    of times, with equal ``rows`` per rank.  ``close()`` is collective too.
    """

    def __init__(self, rows, cols, group=None, lib=None, budget_s=5.0):
        from quantanything_b200 import native

        self.lib = lib or native.get_library()
        self.raw = peer_api(self.lib)
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("the peer gather spans at most 8 GPUs")
        self.rows, self.cols = int(rows), int(cols)
        self.budget_ns = int(budget_s * 1e9)
        self.header = int(self.raw.qa_peer_buffer_header_bytes())
        self.slot_elems = self.world * self.rows * self.cols
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * IPC_HANDLE_BYTES)()
        self._call(self.raw.qa_peer_buffer_create(self.header + 2 * 4 * self.slot_elems,
                                                  ctypes.byref(ptr), handle), "create")
        self.own = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        bases = []
        for r, h in enumerate(handles):
            if r == self.rank:
                bases.append(self.own)
                continue
            buf = (ctypes.c_uint8 * IPC_HANDLE_BYTES).from_buffer_copy(h)
            p = ctypes.c_void_p()
            self._call(self.raw.qa_peer_buffer_open(buf, ctypes.byref(p)), f"open rank {r}")
            self._opened.append(p.value)
            bases.append(p.value)
        self._bases = (ctypes.c_void_p * self.world)(*bases)
        self._views = [torch.as_tensor(
            _DeviceView(self.own + self.header + 4 * s * self.slot_elems,
                        (self.world * self.rows, self.cols)), device="cuda") for s in range(2)]
        self.epoch = 0
        dist.barrier(group=group)  # every rank has mapped every buffer

    def _call(self, rc, what):
        if rc != 0:
            msg = self.lib.raw.qa_last_error().decode(errors="replace")
            self.lib.raw.qa_clear_error()
            raise RuntimeError(f"peer gather {what}: {msg}")

    def __call__(self, q, scale, zp, stream=None):
        if q.dtype != torch.int32 or q.dim() != 2 or tuple(q.shape) != (self.rows, self.cols):
            raise ValueError(f"expected int32 [{self.rows}, {self.cols}], got "
                             f"{q.dtype} {tuple(q.shape)}")
        if q.stride(1) != 1:
            raise ValueError("output rows must be contiguous")
        st = stream or torch.cuda.current_stream()
        self.epoch += 1
        self._call(self.raw.qa_dequantize_gather_peers_dev(
            q.data_ptr(), q.stride(0), int(zp), float(scale), self.rows, self.cols, self._bases,
            self.world, self.rank, self.epoch, self.budget_ns, st.cuda_stream), "launch")
        return self._views[self.epoch & 1]

    def close(self):
        """Collective: unmaps the peers' buffers and frees this rank's."""
        if self.own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # no rank still stores into a buffer
        for p in self._opened:
            self._call(self.raw.qa_peer_buffer_close(p), "close")
        self._opened = []
        self._views = []
        dist.barrier(group=self.group)  # every mapping of this rank's buffer is gone
        self._call(self.raw.qa_peer_buffer_destroy(self.own), "destroy")
        self.own = None


def calibrate_sharded(container, batches, group=None, device=False, lib=None):
    """Each rank calibrates on its shard of ``batches`` (a list of arrays,
    split by index), ranges are all-reduced, then every rank finalizes.

    ``device=True``: each rank's float pass and range reductions run on its
    GPU and the range tables are combined in device memory with one
    all-reduce (``calibrate_device``); ``device`` may also name the torch
    device to use, and ``lib`` the kernel library (tests)."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    mine = [b for i, b in enumerate(batches) if i % world == rank]
    if not mine:
        raise ValueError("fewer calibration batches than ranks")
    if device:
        from quantanything_b200.calibrate_device import calibrate_on_device

        calibrate_on_device(container, mine, reduce_group=group if group is not None else
                            dist.group.WORLD, device=None if device is True else device,
                            lib=lib)
        return container
    container.calibrate(mine, reduce_ranges=lambda r: allreduce_ranges(r, group))
    return container
