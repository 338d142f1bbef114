"""The int16 plane kernels outside the contraction vs the C oracle (B200).

Standalone activation table, Add and Concat rescale (qa_kernels.cpp:307-358),
GlobalAveragePool (quant_layers.py:563-590: int64 sum of centred values,
requantize), the graph-input quantizer (qa_kernels.cpp:363-376) -- each in
its vectorized and its general form -- must equal the oracle bit for bit;
the Softmax float fallback within 1 output LSB.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
QMIN, QMAX = -32768, 32767


@pytest.fixture(scope="module")
def raw(gpu_lib):
    from quantanything_b200.resident import device_api
    from quantanything_b200.resident16 import device_api16

    device_api(gpu_lib)
    return device_api16(gpu_lib)


def _ru(v, m):
    return (v + m - 1) // m * m


def _planes(v, stride):
    """int16 values [rows, C] -> (device buffer, plane distance)."""
    rows, C = v.shape
    plane = _ru(rows * stride, 256)
    full = np.zeros((rows, stride), np.int64)
    full[:, :C] = v
    buf = np.zeros(2 * plane, np.uint8)
    buf[:rows * stride] = (full & 0xFF).astype(np.uint8).ravel()
    buf[plane:plane + rows * stride] = ((full >> 8) & 0xFF).astype(np.uint8).ravel()
    return torch.from_numpy(buf).cuda(), plane


def _values(buf, plane, rows, C, stride):
    b = buf.cpu().numpy()
    lo = b[:rows * stride].reshape(rows, stride)[:, :C].astype(np.int64)
    hi = b[plane:plane + rows * stride].reshape(rows, stride)[:, :C].view(np.int8)
    return lo + 256 * hi.astype(np.int64)


def _ok(lib, rc):
    torch.cuda.synchronize()
    assert rc == 0, lib.raw.qa_last_error().decode()


@pytest.mark.parametrize("C,stride", [(32, 32), (20, 32)])
def test_lut_add_rescale_planes(gpu_lib, oracle, raw, C, stride):
    rng = np.random.default_rng(C)
    rows = 300
    a = rng.integers(QMIN, QMAX + 1, (rows, C))
    b = rng.integers(QMIN, QMAX + 1, (rows, C))
    da, pa = _planes(a, stride)
    db, pb = _planes(b, stride)
    dy, py = _planes(np.zeros((rows, C), np.int64), stride)
    # activation table over the whole int16 range
    table = rng.integers(QMIN, QMAX + 1, 65536).astype(np.int32)
    tdev = torch.from_numpy(table).cuda()
    _ok(gpu_lib, raw.qa_lut16_dev(da.data_ptr(), pa, stride, dy.data_ptr(), py, stride, rows, C,
                                  QMIN, tdev.data_ptr(), 65536, None))
    want = oracle.lut(a.astype(np.int32), table, QMIN)
    np.testing.assert_array_equal(_values(dy, py, rows, C, stride), want)
    # Add (and Sub) with both operands rescaled
    for sign in (1, -1):
        za, zb, zo = 7, -3, 11
        ma, mb = int(rng.integers(2**30, 2**31)), int(rng.integers(2**30, 2**31))
        _ok(gpu_lib, raw.qa_add16_dev(da.data_ptr(), pa, stride, db.data_ptr(), pb, stride,
                                      dy.data_ptr(), py, stride, rows, C, za, ma, 1, zb, mb, 0,
                                      sign, zo, QMIN, QMAX, None))
        want = oracle.add(a.astype(np.int32), b.astype(np.int32), za, ma, 1, zb, mb, 0, zo,
                          QMIN, QMAX, sign=sign)
        np.testing.assert_array_equal(_values(dy, py, rows, C, stride), want)
    # Concat copy: rescale, and the same-grid clip
    m = int(rng.integers(2**30, 2**31))
    _ok(gpu_lib, raw.qa_rescale16_dev(da.data_ptr(), pa, stride, dy.data_ptr(), py, stride,
                                      rows, C, 0, 5, m, 2, -9, QMIN, QMAX, None))
    want = oracle.rescale(a.astype(np.int32), 5, m, 2, -9, QMIN, QMAX)
    np.testing.assert_array_equal(_values(dy, py, rows, C, stride), want)
    _ok(gpu_lib, raw.qa_rescale16_dev(da.data_ptr(), pa, stride, dy.data_ptr(), py, stride,
                                      rows, C, 1, 0, 0, 0, 0, -1000, 1000, None))
    np.testing.assert_array_equal(_values(dy, py, rows, C, stride), np.clip(a, -1000, 1000))


@pytest.mark.parametrize("C,stride", [(64, 64), (24, 32)])
def test_gap_planes(gpu_lib, oracle, raw, C, stride):
    """C % 16 == 0: warp per 16-channel group; else one thread per channel."""
    rng = np.random.default_rng(C + 1)
    N, HW, zp_in = 3, 49, -12
    x = rng.integers(QMIN, QMAX + 1, (N * HW, C))
    dx, px = _planes(x, stride)
    dy, py = _planes(np.zeros((N, C), np.int64), stride)
    m, s = int(rng.integers(2**30, 2**31)), 5
    _ok(gpu_lib, raw.qa_gap16_dev(dx.data_ptr(), px, stride, N, HW, C, zp_in, m, s, 4, QMIN,
                                  QMAX, dy.data_ptr(), py, stride, None))
    acc = (x.reshape(N, HW, C) - zp_in).sum(axis=1)
    want = oracle.requantize(acc.astype(np.int64), N, C, 1, np.full(C, m), np.full(C, s), 4,
                             QMIN, QMAX)
    np.testing.assert_array_equal(_values(dy, py, N, C, stride), want)


@pytest.mark.parametrize("C,H,W,stride", [(3, 12, 16, 4), (5, 7, 9, 16)])
def test_quantize_to_planes(gpu_lib, oracle, raw, C, H, W, stride):
    """stride 4 with H*W % 4 == 0: four pixels per thread; else per byte."""
    rng = np.random.default_rng(H)
    N, scale, zp = 2, 9.155e-05, 3
    x = rng.normal(0, 1.5, (N, C, H, W)).astype(np.float32)
    x[0, 0, 0, :4] = [np.inf, -np.inf, 1e9, -1e9]  # saturation
    x[0, 0, 1, 0] = np.float32(2.5 * scale)         # near a rounding tie
    xd = torch.from_numpy(x).cuda()
    rows = N * H * W
    dy, py = _planes(np.zeros((rows, C), np.int64), stride)
    _ok(gpu_lib, raw.qa_quantize_to_planes16_dev(xd.data_ptr(), dy.data_ptr(), py, N, C, H, W,
                                                 stride, scale, zp, QMIN, QMAX, None))
    want = oracle.quantize_f32(x, scale, zp, QMIN, QMAX)  # NCHW int32
    got = _values(dy, py, rows, stride, stride)
    np.testing.assert_array_equal(got[:, :C].reshape(N, H, W, C).transpose(0, 3, 1, 2), want)
    assert (got[:, C:] == zp).all()  # padding channels hold the zero point


@pytest.mark.parametrize("scale,zp", [(9.155e-05, 3), (1.0 / 32767, 0), (2.5e-05, 32767),
                                      (0.001, -32768), (3e35, 0), (1e-35, 5)])
def test_quantize_to_planes_near_ties(gpu_lib, oracle, raw, scale, zp):
    """The four-pixel kernel rounds inside one FMA and decides the elements
    within 2^-7 of a rounding tie on their own: inputs on and a few ulps
    around every half-integer (k + 1/2) * scale across the int16 range,
    saturating and special values, against the reference's double division.
    The last two scales are outside the float path's range (every element
    takes the division)."""
    rng = np.random.default_rng(abs(zp) + 3)
    with np.errstate(over="ignore"):  # the largest scale overflows float32: +-inf inputs
        k = rng.integers(-70000, 70000, 60000).astype(np.float64)
        ties = ((k + 0.5) * scale).astype(np.float32)
        ulps = rng.integers(-4, 5, ties.size).astype(np.int32)
        near = (ties.view(np.int32) + ulps).view(np.float32)
        ints = (rng.integers(-40000, 40000, 4000) * scale).astype(np.float32)
        rand = (rng.standard_normal(4096) * 20000 * scale).astype(np.float32)
    special = np.array([np.nan, np.inf, -np.inf, 1e30, -1e30, 3.4e38, -3.4e38, 1e-40, -1e-40,
                        0.0, -0.0, 1e-30], np.float32)
    vals = np.concatenate([near, ints, special, rand])
    C, H = 3, 4
    W = -(-vals.size // (C * H))
    W += (-W) % 4
    x = np.zeros(C * H * W, np.float32)
    x[:vals.size] = vals
    x = x.reshape(1, C, H, W)
    xd = torch.from_numpy(x).cuda()
    rows = H * W
    dy, py = _planes(np.zeros((rows, 4), np.int64), 4)
    _ok(gpu_lib, raw.qa_quantize_to_planes16_dev(xd.data_ptr(), dy.data_ptr(), py, 1, C, H, W,
                                                 4, scale, zp, QMIN, QMAX, None))
    want = oracle.quantize_f32(x, scale, zp, QMIN, QMAX)  # NCHW int32 (NaN as x86 leaves it)
    got = _values(dy, py, rows, 4, 4)
    want16 = ((want.reshape(C, rows).T.astype(np.int64) + 32768) & 0xFFFF) - 32768
    np.testing.assert_array_equal(got[:, :C], want16)
    assert (got[:, C] == zp).all()


def test_softmax_planes(gpu_lib, oracle, raw):
    rng = np.random.default_rng(9)
    N, C, stride = 5, 1000, 1008
    x = rng.integers(-3000, 3000, (N, C))
    dx, px = _planes(x, stride)
    in_scale, in_zp, out_scale, out_zp = 0.0021, 4, 1.0 / 32767, 0
    q = torch.empty((N, C), dtype=torch.int32, device="cuda")
    f = torch.empty((N, C), dtype=torch.float32, device="cuda")
    _ok(gpu_lib, raw.qa_softmax16_dev(dx.data_ptr(), px, stride, N, C, in_scale, in_zp,
                                      out_scale, out_zp, QMIN, QMAX, q.data_ptr(), f.data_ptr(),
                                      out_scale, out_zp, None))
    # the reference's fallback: dequantize (float32), float64 softmax with
    # the row max subtracted, float32, qa_quantize_f32
    xf = oracle.dequantize_f32(x.astype(np.int32), in_scale, in_zp).astype(np.float64)
    e = np.exp(xf - xf.max(axis=1, keepdims=True))
    p = (e / e.sum(axis=1, keepdims=True)).astype(np.float32)
    want = oracle.quantize_f32(p, out_scale, out_zp, QMIN, QMAX)
    assert np.abs(q.cpu().numpy().astype(np.int64) - want).max() <= 1
