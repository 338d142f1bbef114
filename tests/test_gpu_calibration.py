"""Calibration through the CUDA library vs the reference's q.json (B200).

QuantContainer.calibrate runs the float graph (quant_container.py:75-91);
its convolutions and GEMMs go through the library's qa_conv_f32 /
qa_gemm_f32 (float_ops.py:160, 175), which run on the GPU here.  On the
reference's own calibration batches (seeded images 100.., as the golden
fixtures were made) every tensor's qparams must match the reference's
q.json up to float32 summation order: the same integer range, the zero
point within 1 and the scale within a relative 1e-4.
"""
import json

import numpy as np
import pytest

from quantanything_b200 import networks
from quantanything_b200.container import QuantContainer
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu
GRAPHS = GOLDEN / "graphs"
# fixture name -> (calibration batches, images per batch), as the fixtures were made
CALIB = {"yolo_mini_int8": (2, 4), "yolo_mini_int16": (2, 4), "yolov8n_cls_int8": (4, 8)}


@pytest.mark.parametrize("name", sorted(CALIB))
def test_gpu_calibration_reproduces_reference_qparams(gpu_lib, name):
    meta = json.loads((GRAPHS / f"{name}.meta.json").read_text())
    g = getattr(networks, meta["builder"])(**meta["kwargs"])
    size = g.inputs[0].shape[2]
    nb, bs = CALIB[name]
    qc = QuantContainer(g, meta["quant_type"], per_channel=True, lib=gpu_lib)
    qc.calibrate([networks.images(bs, size, seed=100 + i) for i in range(nb)])
    ref = json.loads((GRAPHS / f"{name}.qjson").read_text())["qparams"]
    assert set(ref) <= set(qc.qparams)
    worst = 0.0
    for tensor, want in ref.items():
        got = qc.qparams[tensor]
        assert (got.qmin, got.qmax) == (want["qmin"], want["qmax"]), tensor
        assert abs(int(got.zp) - int(want["zp"])) <= 1, tensor
        rel = abs(got.scale - want["scale"]) / abs(want["scale"])
        worst = max(worst, rel)
        assert rel <= 1e-4, (tensor, got.scale, want["scale"])
    assert np.isfinite(worst)


# fixture name -> (calibration batches, images per batch) for the device pass:
# every operator family of the float graphs (ViT: LayerNorm, Softmax, MatMul,
# Gather, Transpose; SPPF: MaxPool; shaping: Pad, Slice, Transpose)
DEVICE_CALIB = dict(CALIB, sppf_mini_int8=(2, 4), shaping_mini_int8=(2, 4),
                    vit_mini_int8=(2, 4), vit_gram_mini_int8=(2, 4), vit_b16_int8=(2, 2))


@pytest.mark.parametrize("name", sorted(DEVICE_CALIB))
def test_device_calibration_reproduces_reference_qparams(gpu_lib, name):
    """The float pass and the range reductions on the GPU
    (QuantContainer.calibrate(..., device=True)) against the reference's
    q.json, with the host calibration's tolerance."""
    meta = json.loads((GRAPHS / f"{name}.meta.json").read_text())
    g = getattr(networks, meta["builder"])(**meta["kwargs"])
    size = meta["image"]
    nb, bs = DEVICE_CALIB[name]
    qc = QuantContainer(g, meta["quant_type"], per_channel=True, lib=gpu_lib)
    qc.calibrate([networks.images(bs, size, seed=100 + i) for i in range(nb)], device=True)
    ref = json.loads((GRAPHS / f"{name}.qjson").read_text())["qparams"]
    assert set(ref) <= set(qc.qparams)
    for tensor, want in ref.items():
        got = qc.qparams[tensor]
        assert (got.qmin, got.qmax) == (want["qmin"], want["qmax"]), tensor
        assert abs(int(got.zp) - int(want["zp"])) <= 1, tensor
        rel = abs(got.scale - want["scale"]) / abs(want["scale"])
        assert rel <= 1e-4, (tensor, got.scale, want["scale"])


def test_device_ranges_match_host_ranges(gpu_lib):
    """Every range the device pass reports against the host float pass
    (NumPy ops around the library's float conv / GEMM) on YOLOv8n-cls: the
    convolutions run the same kernel, so only GEMM sums and float64 library
    functions differ."""
    from quantanything_b200.calibrate_device import DeviceCalibrator

    g = networks.yolov8n_cls()
    batches = [networks.images(4, 224, seed=100 + i) for i in range(2)]
    host = QuantContainer(g, "int8", lib=gpu_lib)
    for b in batches:
        host.run_graph(b, mode="calibrate")
    want = host.get_ranges()
    dev = QuantContainer(g, "int8", lib=gpu_lib)
    cal = DeviceCalibrator(dev)
    for b in batches:
        cal.observe(b)
    got = cal.ranges()
    assert set(got) == set(want)
    for k, (lo, hi) in want.items():
        tol = 1e-5 * max(abs(lo), abs(hi))
        assert abs(got[k][0] - lo) <= tol and abs(got[k][1] - hi) <= tol, (k, got[k], (lo, hi))
