"""Host logic of the device calibration, on the CPU.

DeviceCalibrator walks the graph, derives every launch's shapes, broadcast
strides, layout views, concat offsets and range slots, and decodes the
range table.  Here its kernels are NumPy stand-ins working on the same
pointers (tests/fake_float_kernels.py; convolutions by the C oracle), so
every range it reports must equal the host calibration's (the reference's
float pass: quant_layers.py:130-137, quant_container.py:141-149) up to the
float32 summation order of the stand-ins' GEMMs, and the finalized qparams
must agree the same way.
"""
import numpy as np
import pytest

from quantanything_b200 import networks
from quantanything_b200.calibrate_device import DeviceCalibrator, _fold_dims, calibrate_on_device
from quantanything_b200.container import QuantContainer
from tests.fake_float_kernels import FakeLibrary

GRAPHS = {
    "yolo_mini": lambda: (networks.yolo_mini(width=16), 32),
    "sppf_mini": lambda: (networks.sppf_mini(width=16), 32),
    "bn_mini": lambda: (networks.bn_mini(width=16), 32),
    "mul_mini": lambda: (networks.mul_mini(width=16), 32),
    "shaping_mini": lambda: (networks.shaping_mini(width=16), 32),
    "vit_mini": lambda: (networks.vit(batch=2), 32),
    "vit_gram_mini": lambda: (networks.vit(batch=2, attention="gram"), 32),
}
REL = 2e-6  # float32 GEMM summation order


def _batches(size, n=2, bs=2):
    return [networks.images(bs, size, seed=300 + i) for i in range(n)]


@pytest.mark.parametrize("name", sorted(GRAPHS))
def test_device_ranges_equal_host_ranges(oracle, name):
    g, size = GRAPHS[name]()
    batches = _batches(size)
    host = QuantContainer(g, "int8", lib=oracle)
    for b in batches:
        host.run_graph(b, mode="calibrate")
    want = host.get_ranges()
    dev = QuantContainer(g, "int8", lib=oracle)
    cal = DeviceCalibrator(dev, device="cpu", lib=FakeLibrary(oracle))
    for b in batches:
        cal.observe(b)
    got = cal.ranges()
    assert set(got) == set(want)
    for k, (lo, hi) in want.items():
        glo, ghi = got[k]
        tol = REL * max(abs(lo), abs(hi), 1e-30)
        assert abs(glo - lo) <= tol and abs(ghi - hi) <= tol, (k, (glo, ghi), (lo, hi))


def test_device_calibration_finalizes_like_the_host(oracle):
    g, size = GRAPHS["yolo_mini"]()
    batches = _batches(size)
    host = QuantContainer(g, "int8", lib=oracle)
    host.calibrate(batches)
    dev = QuantContainer(g, "int8", lib=oracle)
    calibrate_on_device(dev, batches, device="cpu", lib=FakeLibrary(oracle))
    assert dev.calibrated and set(dev.qparams) == set(host.qparams)
    for k, qp in host.qparams.items():
        d = dev.qparams[k]
        assert (d.qmin, d.qmax) == (qp.qmin, qp.qmax)
        assert abs(int(d.zp) - int(qp.zp)) <= 1
        assert abs(d.scale - qp.scale) <= 1e-5 * qp.scale


def test_ranges_accumulate_over_batches_and_skip_unobserved(oracle):
    g, size = GRAPHS["yolo_mini"]()
    qc = QuantContainer(g, "int8", lib=oracle)
    cal = DeviceCalibrator(qc, device="cpu", lib=FakeLibrary(oracle))
    assert cal.ranges() == {}
    a, b = _batches(size)
    cal.observe(a)
    first = cal.ranges()
    cal.observe(b)
    both = cal.ranges()
    for k in first:
        assert both[k][0] <= first[k][0] and both[k][1] >= first[k][1]


def test_nan_in_a_calibration_tensor_is_reported(oracle):
    g, size = GRAPHS["yolo_mini"]()
    qc = QuantContainer(g, "int8", lib=oracle)
    cal = DeviceCalibrator(qc, device="cpu", lib=FakeLibrary(oracle))
    x = _batches(size, n=1)[0]
    x[0, 0, 0, 0] = np.nan
    cal.observe(x)
    with pytest.raises(ValueError, match="NaN"):
        cal.ranges()


def test_fold_dims_merges_contiguous_runs():
    # a dense [2, 3, 4] copy is one run of 24
    assert _fold_dims((2, 3, 4), (12, 4, 1), (12, 4, 1)) == ([24], [[1], [1]])
    # a [0, 2, 1] transpose keeps its three dimensions
    assert _fold_dims((2, 4, 3), (12, 1, 4), (12, 3, 1)) == ([2, 4, 3], [[12, 1, 4], [12, 3, 1]])
    # broadcasting a channel vector over [2, 8, 5, 5]: the spatial run folds
    shape, (a, b) = _fold_dims((2, 8, 5, 5), (200, 25, 5, 1), (0, 1, 0, 0))
    assert shape == [2, 8, 25] and a == [200, 25, 1] and b == [0, 1, 0]
