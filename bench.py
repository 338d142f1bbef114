#!/usr/bin/env python
"""Benchmark: int8 YOLOv8n-cls integer inference, images/sec on B200.

Workload (configuration 2): YOLOv8n-cls, random init (He-normal convs with a
folded random BatchNorm), int8 per-channel weights, int8 activations with the
qparams the reference's QuantContainer calibrated on 32 seeded images
(tests/golden/graphs/yolov8n_cls_int8.qjson), batch 64 per GPU of N(0,1)
images clipped to +-3 (synthetic: no dataset is reachable).

One step = one integer forward pass over one batch of 64 images per GPU:
graph-input quantization, 26 fused conv layers, GAP, Gemm 1280->1000 and
the Softmax float fallback, captured in a CUDA graph.

  value  -- images/s with the batch already in HBM, device time from CUDA
            events around each step; L2 flushed (256 MiB write) between
            steps, outside the events; max over ranks.
  e2e    -- images/s through the public host-to-host call
            (ResidentNet.run_pipelined): pinned host images -> device,
            forward, float32 probabilities -> host, every step's copies
            inside the events; a step's host->device copy overlaps the
            previous step's forward.
  e2e_dropin -- images/s of the drop-in route: the reference's layer-by-layer
            execution driving the CUDA library's host-pointer ABI
            (one H2D/D2H per layer), wall clock.
  roofline -- dominant kernel of the step, measured live with CUDA events:
            a CUDA graph of ten (L2 flush, step) rounds against one of the
            ten flushes alone (the single-replay figure beside it).
  cpu_baseline -- the reference's own C++ kernels (oracle/_ref, OpenMP, all
            host threads) driven layer by layer, on a bounded sample.

--impl reference runs only that CPU reference arm (rank 0; other ranks exit).

--workload vit_b16 measures configuration 3 instead: ViT-B/16 (trunc-normal
0.02 random init), int8, batch 256 per GPU, with the reference-calibrated
q.json of tests/golden/graphs/vit_b16_int8.qjson, on the same contract.
--workload yolov8n_cls_int16 measures configuration 4: the same YOLOv8n-cls
graph quantized int16 (tests/golden/graphs/yolov8n_cls_int16.qjson, every
Conv / Gemm on the reference's int64-accumulator route), batch 1024 per GPU,
run by the 16-bit resident executor (byte-split tensor-core contractions).
"""

import argparse
import hashlib
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

GRAPHS = REPO / "tests" / "golden" / "graphs"
REF_LIB = REPO / "oracle" / "_ref" / "libqa_kernels_ref.so"
UNIT = "images/s"
IMAGE = 224
_VIT_B16 = {"img": 224, "patch": 16, "dim": 768, "heads": 12, "depth": 12, "classes": 1000,
            "std": 0.02}

def _graph(kind, batch):
    """The workload's graph (a ViT graph holds its batch in its Reshapes)."""
    from quantanything_b200 import networks

    if kind == "vit_b16":
        return networks.vit(batch=batch, **_VIT_B16)
    return networks.yolov8n_cls()


# workload name -> metric, q.json, graph for a batch, per-GPU batch, CPU sample batch
WORKLOADS = {
    "yolov8n_cls": {
        "metric": "int8 YOLOv8n-cls images/sec", "qjson": GRAPHS / "yolov8n_cls_int8.qjson",
        "graph": lambda b: _graph("yolov8n_cls", b),
        "batch": 64, "cpu_batch": 64, "ref_batch": 64, "classes": 1000,
        "calib": (4, 8),
        "name": "cfg2: YOLOv8n-cls int8 integer inference (random init, BN folded, "
                "reference-calibrated q.json)"},
    "yolov8n_cls_int16": {
        "metric": "int16 YOLOv8n-cls images/sec", "qjson": GRAPHS / "yolov8n_cls_int16.qjson",
        "graph": lambda b: _graph("yolov8n_cls", b), "dtype": "int16",
        "batch": 1024, "cpu_batch": 16, "ref_batch": 32, "classes": 1000,
        "name": "cfg4: YOLOv8n-cls int16 integer inference (random init, BN folded, "
                "reference-calibrated q.json; every Conv / Gemm on the reference's wide "
                "int64-accumulator route)"},
    "vit_b16": {
        "metric": "int8 ViT-B/16 images/sec", "qjson": GRAPHS / "vit_b16_int8.qjson",
        "graph": lambda b: _graph("vit_b16", b),
        "batch": 256, "cpu_batch": 1, "ref_batch": 2, "classes": 1000,
        "name": "cfg3: ViT-B/16 int8 integer inference (random init, reference-calibrated "
                "q.json; LayerNorm / attention float fallbacks on the GPU)"},
}
W = WORKLOADS["yolov8n_cls"]
METRIC = W["metric"]
PER_GPU_BATCH = W["batch"]


def select_workload(name):
    global W, METRIC, PER_GPU_BATCH
    W = WORKLOADS[name]
    METRIC, PER_GPU_BATCH = W["metric"], W["batch"]


def in_graph_ms(launch, flush, repeat=10, reps=5):
    """Device time (ms) of one launch of ``launch(stream_handle)``: a CUDA
    graph of ``repeat`` rounds of (zero ``flush``, launch) against one of the
    ``repeat`` flushes alone, the difference of the medians of ``reps``
    replays over ``repeat`` (single launches between CUDA events carry the
    launch and the events' 2.048 us timestamp grid on B200)."""
    import torch

    s = torch.cuda.Stream(flush.device)
    g0, g1 = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g0, stream=s):
            for _ in range(repeat):
                flush.zero_()
        with torch.cuda.graph(g1, stream=s):
            for _ in range(repeat):
                flush.zero_()
                launch(s.cuda_stream)
    torch.cuda.synchronize(flush.device)

    def replay_ms(g):
        with torch.cuda.stream(s):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(s)
            g.replay()
            e1.record(s)
        e1.synchronize()
        return e0.elapsed_time(e1)

    t1, t0 = [], []
    for _ in range(reps):
        t1.append(replay_ms(g1))
        t0.append(replay_ms(g0))
    del g0, g1
    return max(float(np.median(t1) - np.median(t0)), 0.0) / repeat


def measure_fused_configs(dev, stream, flush, peak_tops, reps=10):
    """cfg0 (Linear 256x768x3072) and cfg1 (conv 3x3 [32,64,56,56] -> 128 with
    the SiLU table) on the fused int8 tensor-core kernel, device-resident:
    the in-graph launch time (``in_graph_ms``, L2 flushed before each
    launch) and, beside it, the median CUDA-event time of single launches,
    L2 flushed before each one."""
    import torch

    from quantanything_b200 import native
    from quantanything_b200.fused_cases import FusedCase

    res = {}
    for name, shape in (("cfg0", "Linear [256, 768] x [768, 3072], int8 out"),
                        ("cfg1", "conv 3x3 [32, 64, 56, 56] * [128, 64, 3, 3] + SiLU table")):
        case = FusedCase(native.get_library(), name, dev)
        for _ in range(3):
            case.launch(stream.cuda_stream)
        times = []
        for _ in range(reps):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            case.launch(stream.cuda_stream)
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        t1 = float(np.median(times)) / 1e3
        t = in_graph_ms(case.launch, flush) / 1e3
        tops = case.ops / t / 1e12
        res[name] = {"shape": shape, "us": round(t * 1e6, 2), "TOPS": round(tops, 1),
                     "frac": round(tops / peak_tops, 4), "block_n": int(case.desc.block_n),
                     "us_single_launch": round(t1 * 1e6, 2),
                     "frac_single_launch": round(case.ops / t1 / 1e12 / peak_tops, 4)}
    res["peak_TOPS"] = peak_tops
    res["timing"] = ("in-graph: (10 x (L2 flush + launch) - 10 x flush) / 10, median of 5; "
                     f"*_single_launch: median of {reps} single launches between CUDA events, "
                     "L2 flushed before each")
    return res


def measure_elementwise(dev, stream, flush, hbm_peak, reps=5):
    """The standalone memory-bound resident kernels on tensors larger than
    L2 (2^21 pixels x 64 channels: 128 MiB per 8-bit operand): median
    CUDA-event time of single launches, L2 flushed before each; algorithmic
    bytes = every operand read once plus the output written once.

    Two timings per kernel: after the flush alone (a zero fill of a buffer
    larger than L2, whose dirty lines the kernel's own misses then write
    back to DRAM during the timed launch), and with L2 clean (the same fill
    followed, outside the events, by a read of another buffer larger than
    L2, which writes those lines back first): the second is the kernel's
    own DRAM traffic, as an ncu capture with its cache control sees it."""
    import ctypes

    import torch

    from quantanything_b200 import native
    from quantanything_b200.resident import device_api

    lib = native.get_library()
    raw = device_api(lib)
    st = ctypes.c_void_p(stream.cuda_stream)
    rows, C = 1 << 21, 64
    n = rows * C
    a = torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev)
    b = torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev)
    y = torch.empty(n, dtype=torch.uint8, device=dev)
    tab = torch.randint(-128, 128, (256,), dtype=torch.int32, device=dev)
    acc = torch.randint(-(2**20), 2**20, (n,), dtype=torch.int32, device=dev)
    q32 = torch.empty(n, dtype=torch.int32, device=dev)
    mult = torch.full((C,), 1 << 30, dtype=torch.int64, device=dev)
    shift = torch.full((C,), 4, dtype=torch.int64, device=dev)
    img = torch.randn(2048, 3, 64, 64, device=dev)  # 2^23 pixels: 100 MB, past L2
    clean = torch.ones(flush.numel(), dtype=torch.uint8, device=dev)  # read-only after this
    m30 = 1 << 30
    cases = {
        "lut (table)": (2 * n, lambda: raw.qa_lut_bytes_dev(a.data_ptr(), C, 1, y.data_ptr(), C,
                                                           rows, C, -128, tab.data_ptr(), 256, st)),
        "rescale": (2 * n, lambda: raw.qa_rescale_bytes_dev(a.data_ptr(), C, 1, y.data_ptr(), C,
                                                            rows, C, 0, 3, m30, 1, -4, -128, 127,
                                                            st)),
        "add": (3 * n, lambda: raw.qa_add_bytes_dev(a.data_ptr(), C, 1, b.data_ptr(), C, 1,
                                                    y.data_ptr(), C, rows, C, 5, m30, 1, -2, m30,
                                                    1, 1, 7, -128, 127, st)),
        "mul": (3 * n, lambda: raw.qa_mul_bytes_dev(a.data_ptr(), C, 1, b.data_ptr(), C, 1,
                                                    y.data_ptr(), C, rows, C, 3, -1, m30, 6, 2,
                                                    -128, 127, st)),
        "maxpool k5 s1 p2": (2 * n, lambda: raw.qa_maxpool_bytes_dev(
            a.data_ptr(), C, 1, y.data_ptr(), C, 512, 64, 64, C, 5, 5, 1, 1, 2, 2, 1, 1, 64, 64,
            -128, st)),
        "gap 49 px": (n + n // 49, lambda: raw.qa_gap_dev(
            a.data_ptr(), C, 1, rows // 49, 49, C, 0, m30, 5, 0, -128, 127, y.data_ptr(), C, st)),
        "requantize i32 -> i32": (8 * n, lambda: raw.qa_requantize_i32_dev(
            acc.data_ptr(), q32.data_ptr(), rows, C, 1, mult.data_ptr(), shift.data_ptr(), None,
            None, 0, -128, 127, st)),
        "requantize i32 -> i32, NCHW (inner 4096)": (8 * n, lambda: raw.qa_requantize_i32_dev(
            acc.data_ptr(), q32.data_ptr(), rows // 4096, C, 4096, mult.data_ptr(),
            shift.data_ptr(), None, None, 0, -128, 127, st)),
        "quantize f32 -> nhwc": (img.numel() * 4 + 4 * rows * 4,
                                 lambda: raw.qa_quantize_to_nhwc_dev(
                                     img.data_ptr(), y.data_ptr(), 2048, 3, 64, 64, 4, 0.0235, 0,
                                     -128, 127, st)),
    }
    res = {}
    for name, (nbytes, fn) in cases.items():
        for _ in range(2):
            if fn() != 0:
                raise RuntimeError(f"{name}: {lib.raw.qa_last_error().decode()}")
        times, times_clean = [], []
        for _ in range(reps):
            for clean_l2 in (False, True):
                flush.zero_()
                if clean_l2:
                    torch.amax(clean)
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                fn()
                e1.record(stream)
                e1.synchronize()
                (times_clean if clean_l2 else times).append(e0.elapsed_time(e1))
        t = float(np.median(times)) / 1e3
        tc = float(np.median(times_clean)) / 1e3
        gbs, gbs_c = nbytes / t / 1e9, nbytes / tc / 1e9
        res[name] = {"us": round(t * 1e6, 1), "GB/s": round(gbs, 1),
                     "frac": round(gbs / hbm_peak, 4), "bytes": int(nbytes),
                     "us_clean_l2": round(tc * 1e6, 1),
                     "frac_clean_l2": round(gbs_c / hbm_peak, 4)}
    res["timing"] = (f"median of {reps} single launches on 2^21 pixels x 64 channels (the "
                     "float quantizer: 2^23 pixels x 3 channels), L2 flushed before each (a zero "
                     "fill larger than L2; its dirty lines are written back during the launch); "
                     "*_clean_l2: the fill then a read of another buffer larger than L2, outside "
                     "the events, so only the kernel's own traffic is timed; bytes = operands "
                     "read once + output written once")
    return res


def calibrate_over_nccl(world):
    """Sharded calibration of the workload's graph over the process group
    (each rank runs the float graph on its share of the reference's
    calibration images on its GPU, every range folded on the device, then
    one all-reduce of the device range tables), compared with the
    reference-calibrated q.json the timed forward uses.  Outside every
    timed region."""
    import torch
    import torch.distributed as dist

    from quantanything_b200 import distributed, networks
    from quantanything_b200.container import QuantContainer

    nb, bs = W["calib"]
    images = [networks.images(bs, IMAGE, seed=100 + i) for i in range(nb)]
    batches = [x[j:j + 1] for x in images for j in range(bs)]  # one image per batch
    qc = QuantContainer(W["graph"](1), W.get("dtype", "int8"), per_channel=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    distributed.calibrate_sharded(qc, batches, device=True)
    dt = time.perf_counter() - t0
    ref = json.loads(Path(W["qjson"]).read_text())["qparams"]
    rel = max(abs(qc.qparams[k].scale - v["scale"]) / abs(v["scale"]) for k, v in ref.items())
    dzp = max(abs(int(qc.qparams[k].zp) - int(v["zp"])) for k, v in ref.items())
    return {"backend": dist.get_backend(), "ranks": dist.get_world_size(),
            "float_pass": "device (qa_f32_* kernels; ranges folded on the GPU, one all-reduce "
                          "of the range tables)",
            "images": nb * bs, "tensors": len(ref), "seconds": round(dt, 3),
            "max_rel_scale_diff_vs_qjson": float(f"{rel:.3g}"), "max_zp_diff_vs_qjson": dzp}


def config(world, extra=None):
    c = {"workload": W["name"],
         "global_batch": PER_GPU_BATCH * world, "per_gpu_batch": PER_GPU_BATCH,
         "image": [3, IMAGE, IMAGE], "parallelism": f"dp{world} (batch-sharded replicas)",
         "l2": "flushed with a 256 MiB write between timed steps (outside the events)"}
    if extra:
        c.update(extra)
    return c


# ------------------------------------------------------------ CPU arms --
def cpu_reference_sample(seconds, images_per_step, steps=None):
    """The reference's C++ kernels (OpenMP) driven layer by layer; returns
    (images/s, threads, sample description, per-step seconds list)."""
    from quantanything_b200 import networks
    from quantanything_b200.container import QuantContainer
    from quantanything_b200.native import KernelLibrary

    if not REF_LIB.exists():
        raise FileNotFoundError(f"{REF_LIB} missing (built by __graft_entry__.build())")
    threads = len(os.sched_getaffinity(0))
    os.environ["OMP_NUM_THREADS"] = str(threads)
    lib = KernelLibrary(REF_LIB)
    lib.set_num_threads(threads)
    qc = QuantContainer.load(W["graph"](images_per_step), W["qjson"], lib=lib)
    x = networks.images(images_per_step, IMAGE, seed=2024)
    qc.run_graph(x, "integer")  # warm caches / thread pool
    times = []
    t_end = time.perf_counter() + seconds
    while (steps is None and (not times or time.perf_counter() < t_end)) or (
            steps is not None and len(times) < steps):
        t0 = time.perf_counter()
        qc.run_graph(x, "integer")
        times.append(time.perf_counter() - t0)
    ips = images_per_step * len(times) / sum(times)
    sample = (f"{len(times)} step(s) of {images_per_step} images through the reference's "
              f"qa_kernels.cpp (OpenMP, {lib.num_threads()} threads) driven layer by layer")
    return ips, lib.num_threads(), sample, times


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    images = W["ref_batch"]  # enough work per step for every host thread
    ips, threads, sample, times = cpu_reference_sample(0, images, steps=args.warmup)
    ips, threads, sample, times = cpu_reference_sample(0, images, steps=args.steps)
    ms = 1000.0 * sum(times) / len(times)
    line = {"impl": "reference", "metric": METRIC, "value": round(ips, 3), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": W.get("dtype", "int8"),
            "data": "synthetic N(0,1) images, random init",
            "config": config(world, {"reference_step": f"{images} images per step on the "
                                                       "host CPU"}),
            "cpu_baseline": {"value": round(ips, 3), "unit": UNIT, "cores": threads,
                             "kind": "reference", "sample": sample},
            "e2e": {"value": round(ips, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# -------------------------------------------------------------- clocks --
class ClockSampler:
    """Samples SM clock, power and clock-event reasons through NVML."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, index, period_s=0.005):
        self.index, self.period = index, period_s
        self.samples, self._stop = [], threading.Event()
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # NVML missing: report no clocks rather than fail
            self.max_mhz = None

    def _reasons(self):
        nv = self.nv
        fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or getattr(
            nv, "nvmlDeviceGetCurrentClocksThrottleReasons")
        return fn(self.h)

    def _loop(self):
        while not self._stop.is_set():
            try:
                self.samples.append((self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM),
                                     self._reasons()))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._loop, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [m for m, _ in self.samples]
        bits = 0
        for _, r in self.samples:
            bits |= int(r)
        names = [n for b, n in self.REASONS.items() if bits & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], 2.0 * d["bf16_tflops"], "measured"
    return 6650.0, 2.0 * 1590.0, "fallback"


# ---------------------------------------------------------------- main --
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-dropin", action="store_true")
    ap.add_argument("--workload", default="yolov8n_cls", choices=sorted(WORKLOADS))
    ap.add_argument("--profile-forwards", type=int, default=0,
                    help="run this many plain forward passes of the workload and exit "
                         "(the command the ncu summaries under profiles/ are taken with)")
    ap.add_argument("--profile-fused", choices=["cfg0", "cfg1"], default=None,
                    help="launch the fused int8 kernel on this kernel-level configuration "
                         "three times and exit (for ncu captures)")
    ap.add_argument("--profile-elementwise", action="store_true",
                    help="run the standalone memory-bound kernels of the bench line's "
                         "'elementwise' entry once each and exit (for ncu captures)")
    ap.add_argument("--batch", type=int, default=None,
                    help="per-GPU batch of a --profile-forwards run (the bench line itself "
                         "always uses the workload's configured batch)")
    args = ap.parse_args()
    select_workload(args.workload)
    if args.batch is not None:
        if not args.profile_forwards:
            ap.error("--batch only applies to --profile-forwards runs")
        global PER_GPU_BATCH
        PER_GPU_BATCH = args.batch
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.profile_fused:
        import torch

        from quantanything_b200 import native
        from quantanything_b200.fused_cases import FusedCase

        case = FusedCase(native.get_library(), args.profile_fused, torch.device("cuda", local))
        for _ in range(3):
            case.launch(torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        print(json.dumps({"profile_fused": args.profile_fused, "launches": 3}))
        return
    if args.profile_elementwise:
        import torch

        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        res = measure_elementwise(dev, torch.cuda.current_stream(dev), flush, peaks()[0], reps=1)
        print(json.dumps({"profile_elementwise": {k: v for k, v in res.items()
                                                  if isinstance(v, dict)}}))
        return
    args.warmup = max(args.warmup, 3)

    import torch

    from quantanything_b200 import networks
    from quantanything_b200.container import QuantContainer
    from quantanything_b200.resident import ResidentNet

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    from quantanything_b200 import native

    native.get_library().set_device(local)  # library work on this rank's GPU
    qc = QuantContainer.load(W["graph"](PER_GPU_BATCH), W["qjson"])
    if args.workload == "vit_b16":
        from quantanything_b200.resident_vit import ResidentViT

        net = ResidentViT(qc, PER_GPU_BATCH, dev)
    elif W.get("dtype") == "int16":
        from quantanything_b200.resident16 import ResidentNet16

        net = ResidentNet16(qc, PER_GPU_BATCH, dev)
    else:
        net = ResidentNet(qc, PER_GPU_BATCH, dev)
    x_host = networks.images(PER_GPU_BATCH, IMAGE, seed=1000 + rank)
    x_pinned = torch.from_numpy(x_host).pin_memory()
    out_pinned = torch.empty((PER_GPU_BATCH, W["classes"]), dtype=torch.float32).pin_memory()
    net.x_dev.copy_(x_pinned)
    if args.profile_forwards:
        for _ in range(args.profile_forwards):
            net.forward_device()
        torch.cuda.synchronize(dev)
        net.check_status()
        print(json.dumps({"profile_forwards": args.profile_forwards, "launches_per_forward":
                          len(net.steps)}))
        return
    calibration = None
    if dist is not None and "calib" in W:
        calibration = calibrate_over_nccl(world)
    net.capture()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- value: device-resident forward, CUDA-graph replay per step
    for _ in range(args.warmup):
        net.replay()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    with ClockSampler(local) as clocks:
        for k in range(args.steps):
            flush.zero_()
            starts[k].record(stream)
            net.replay()
            ends[k].record(stream)
        barrier()
    elapsed_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    net.check_status()
    elapsed_ms = max_over_ranks(elapsed_ms)
    value = world * PER_GPU_BATCH * args.steps / (elapsed_ms / 1e3)

    # ---- e2e: pinned host images in, probabilities out, every step, through
    # the public pipelined call (each step's host->device copy overlaps the
    # previous step's forward; every copy is inside the timed region).  With
    # several ranks every step also gathers the whole batch's probabilities
    # on every rank -- the output dequantize fused with the gather, one
    # kernel per rank storing its rows into every rank's buffer over NVLink
    # peer memory -- and copies the whole batch out.
    e2e_steps = max(min(args.steps, 50), 1)
    collect = None
    gather = None
    if dist is not None:
        from quantanything_b200 import distributed

        gather = distributed.PeerGather(PER_GPU_BATCH, W["classes"])
        out_qp = net.output_qparams()
        out_pinned = torch.empty((world * PER_GPU_BATCH, W["classes"]),
                                 dtype=torch.float32).pin_memory()

        def collect(y):
            return gather(net.output_int(), out_qp.scale, out_qp.zp)

    net.run_pipelined([x_pinned] * 3, [out_pinned] * 3, collect)
    es = torch.cuda.Event(enable_timing=True)
    ee = torch.cuda.Event(enable_timing=True)
    barrier()
    es.record(stream)
    net.run_pipelined([x_pinned] * e2e_steps, [out_pinned] * e2e_steps, collect)
    ee.record(stream)
    barrier()
    e2e_ms = max_over_ranks(es.elapsed_time(ee))
    e2e = world * PER_GPU_BATCH * e2e_steps / (e2e_ms / 1e3)
    gather_ok = None
    if gather is not None:
        net.check_status()  # a gather wait that ran out is reported here
        # the last step's gathered batch: this rank's rows equal its own
        # dequantized output, and every rank holds the same bytes
        own = torch.equal(out_pinned[rank * PER_GPU_BATCH:(rank + 1) * PER_GPU_BATCH],
                          net.out_f32.cpu())
        digest = float(int.from_bytes(
            hashlib.sha1(out_pinned.numpy().tobytes()).digest()[:6], "little"))
        same = max_over_ranks(digest) == -max_over_ranks(-digest)
        gather_ok = max_over_ranks(0.0 if own else 1.0) == 0.0 and same

    # ---- roofline of the dominant kernel: every step timed inside a CUDA
    # graph of ten (L2 flush, step) rounds against a graph of the ten flushes
    # alone (no host launch work; the event granularity and the graph launch
    # spread over ten launches); the single-replay figure of the dominant
    # step (one graph launch per event pair) is reported beside it
    step_ms = net.time_steps_in_graph(flush)
    single_ms = net.time_steps_graphed(reps=20, flush=flush)
    costs = net.step_costs()
    dom = int(np.argmax(step_ms))
    label, dom_bytes, dom_ops = costs[dom]
    hbm_peak, int8_peak_tops, peak_kind = peaks()
    # 16-bit contractions issue four 8-bit tensor-core products per MAC
    tensor_peak = int8_peak_tops / 4 if W.get("dtype") == "int16" else int8_peak_tops
    tensor_note = ("; int16 tensor = int8 / 4 (byte-split: four int8 MMAs per int16 MAC)"
                   if W.get("dtype") == "int16" else "")
    dur_s = step_ms[dom] / 1e3
    ai = dom_ops / max(dom_bytes, 1)
    ridge = tensor_peak * 1e12 / (hbm_peak * 1e9)
    traffic = None
    tfile = REPO / "profiles" / "dram_traffic.json"
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get(label)
    if ai < ridge:
        achieved = dom_bytes / dur_s / 1e9
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak,
                    "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                    "traffic": traffic, "algorithmic_bytes": int(dom_bytes)}
    else:
        achieved = dom_ops / dur_s / 1e12
        roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": tensor_peak,
                    "unit": "TOPS", "frac": round(achieved / tensor_peak, 4),
                    "traffic": traffic, "algorithmic_ops": int(dom_ops)}
    roofline.update({"kernel": label, "us_per_launch": round(step_ms[dom] * 1e3, 2),
                     "us_per_launch_single_replay": round(single_ms[dom] * 1e3, 2),
                     "timing": "in-graph: (10 x (L2 flush + launch) - 10 x flush) / 10, median "
                               "of 5; single replay: one graph launch of the step per CUDA-event "
                               "pair, L2 flushed before each (its figures fall on a 2.048 us "
                               "grid and carry the graph launch)",
                     "share_of_step": round(float(step_ms[dom] / step_ms.sum()), 4),
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json; int8 tensor = 2 x "
                                    f"measured bf16 cuBLAS{tensor_note})"})
    kernels = [{"kernel": c[0], "us": round(float(t) * 1e3, 2),
                "GB/s": round(c[1] / (t / 1e3) / 1e9, 1),
                "TOPS": round(c[2] / (t / 1e3) / 1e12, 2) if c[2] else 0.0}
               for c, t in zip(costs, step_ms)]

    # all contraction launches of the step against the int8 tensor peak
    con = [(c, float(t)) for c, t in zip(costs, step_ms) if c[2]]
    con_ms = sum(t for _, t in con)
    con_tops = sum(c[2] for c, _ in con) / (con_ms / 1e3) / 1e12
    contractions = {"launches": len(con), "us": round(con_ms * 1e3, 1),
                    "achieved": round(con_tops, 1), "peak": tensor_peak, "unit": "TOPS",
                    "frac": round(con_tops / tensor_peak, 4)}
    fused_gemm = measure_fused_configs(dev, stream, flush, int8_peak_tops)
    elementwise = measure_elementwise(dev, stream, flush, hbm_peak)

    # ---- drop-in ABI route (rank 0, N=1) and CPU baseline
    dropin = cpu = None
    if rank == 0 and world == 1 and not args.no_dropin:
        nb = PER_GPU_BATCH if args.workload == "yolov8n_cls" else W["ref_batch"]
        qd = qc if nb == PER_GPU_BATCH else QuantContainer.load(W["graph"](nb), W["qjson"])
        qd.run_graph(x_host[:nb], "integer")
        t0 = time.perf_counter()
        qd.run_graph(x_host[:nb], "integer")
        dt = time.perf_counter() - t0
        dropin = {"value": round(nb / dt, 2), "unit": UNIT,
                  "route": "layer-by-layer host-pointer ABI (QA_LIB drop-in), wall clock, "
                           f"{nb} images"}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ips, threads, sample, _ = cpu_reference_sample(args.cpu_seconds, W["cpu_batch"])
        cpu = {"value": round(ips, 3), "unit": UNIT, "cores": threads, "kind": "reference",
               "sample": sample}

    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(elapsed_ms / args.steps, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": W.get("dtype", "int8"),
                "data": "synthetic N(0,1) images clipped to +-3, random-init weights",
                "config": config(world),
                "e2e": {"value": round(e2e, 1), "unit": UNIT,
                        "h2d_bytes_per_step": int(x_pinned.numel() * 4),
                        "d2h_bytes_per_step": int(out_pinned.numel() * 4)},
                "roofline": roofline, "cpu_baseline": cpu, "clocks": clocks.summary(),
                "gpu_launches": int(net.launch_count * args.steps),
                "launches_per_step": net.launch_count, "contractions": contractions,
                "fused_gemm": fused_gemm, "elementwise": elementwise, "kernels": kernels}
        if dropin:
            line["e2e_dropin"] = dropin
        if dist is not None:
            line["collectives"] = {
                "backend": dist.get_backend(), "nccl_ranks": world,
                "e2e_gather": f"qa_dequantize_gather_peers_dev: each rank's int32 [{PER_GPU_BATCH}, "
                              f"{W['classes']}] output dequantized and stored into every rank's "
                              "buffer over NVLink peer memory, one kernel per rank per step, "
                              "inside the e2e region",
                "calibration_allreduce": calibration,
                "gather_matches_local_dequantize": gather_ok}
        print(json.dumps(line), flush=True)
    del net._graph
    if gather is not None:
        net.check_status()
        gather.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
