"""The standalone 8-bit resident layers vs the C oracle (B200).

Activation table, Concat rescale / clip, Add / Sub, Mul (qa_kernels.cpp:
307-358) and MaxPool padded with qmin (quant_layers.py:647-648) on NHWC byte
views -- in their 16-channel vector form (C and strides multiples of 16)
and their per-byte form -- must equal the reference's integer results bit
for bit, for signed and unsigned bytes.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
CASES = [(32, 32, 1), (32, 48, 0), (24, 32, 1), (24, 24, 0)]  # (C, pixel stride, signed)


@pytest.fixture(scope="module")
def raw(gpu_lib):
    from quantanything_b200.resident import device_api

    return device_api(gpu_lib)


def _dev(v, stride, signed):
    rows, C = v.shape
    full = np.zeros((rows, stride), np.int64)
    full[:, :C] = v
    return torch.from_numpy((full & 0xFF).astype(np.uint8).ravel()).cuda()


def _host(buf, rows, C, stride, signed):
    b = buf.cpu().numpy().reshape(rows, stride)[:, :C]
    return (b.view(np.int8) if signed else b).astype(np.int64)


def _vals(rng, shape, signed):
    return rng.integers(-128, 128, shape) if signed else rng.integers(0, 256, shape)


def _ok(lib, rc):
    torch.cuda.synchronize()
    assert rc == 0, lib.raw.qa_last_error().decode()


@pytest.mark.parametrize("C,stride,signed", CASES)
def test_byte_layers(gpu_lib, oracle, raw, C, stride, signed):
    rng = np.random.default_rng(C * 7 + stride + signed)
    rows = 257
    qmin, qmax = (-128, 127) if signed else (0, 255)
    a, b = _vals(rng, (rows, C), signed), _vals(rng, (rows, C), signed)
    da, db = _dev(a, stride, signed), _dev(b, stride, signed)
    dy = torch.zeros(rows * stride, dtype=torch.uint8, device="cuda")
    a32, b32 = a.astype(np.int32), b.astype(np.int32)

    def got():
        return _host(dy, rows, C, stride, signed)

    table = rng.integers(qmin, qmax + 1, 256).astype(np.int32)
    tdev = torch.from_numpy(table).cuda()
    _ok(gpu_lib, raw.qa_lut_bytes_dev(da.data_ptr(), stride, signed, dy.data_ptr(), stride, rows,
                                      C, qmin, tdev.data_ptr(), 256, None))
    np.testing.assert_array_equal(got(), oracle.lut(a32, table, qmin))

    m = int(rng.integers(2**30, 2**31))
    _ok(gpu_lib, raw.qa_rescale_bytes_dev(da.data_ptr(), stride, signed, dy.data_ptr(), stride,
                                          rows, C, 0, 3, m, 1, -4 if signed else 9, qmin, qmax,
                                          None))
    np.testing.assert_array_equal(got(), oracle.rescale(a32, 3, m, 1, -4 if signed else 9,
                                                        qmin, qmax))
    _ok(gpu_lib, raw.qa_rescale_bytes_dev(da.data_ptr(), stride, signed, dy.data_ptr(), stride,
                                          rows, C, 1, 0, 0, 0, 0, qmin + 20, qmax - 20, None))
    np.testing.assert_array_equal(got(), np.clip(a, qmin + 20, qmax - 20))

    # Add / Sub; the last case's terms pass 2^61 (the 128-bit per-element path)
    for ma, sa, sign in ((int(rng.integers(2**30, 2**31)), 1, 1),
                         (int(rng.integers(2**30, 2**31)), 0, -1), (2**62 - 1, -31, 1)):
        mb = int(rng.integers(2**30, 2**31))
        _ok(gpu_lib, raw.qa_add_bytes_dev(da.data_ptr(), stride, signed, db.data_ptr(), stride,
                                          signed, dy.data_ptr(), stride, rows, C, 5, ma, sa, -2,
                                          mb, 1, sign, 7, qmin, qmax, None))
        want = oracle.add(a32, b32, 5, ma, sa, -2, mb, 1, 7, qmin, qmax, sign=sign)
        np.testing.assert_array_equal(got(), want)

    for mm, ss in ((int(rng.integers(2**30, 2**31)), 6), (2**40, -3)):  # 64-bit / 128-bit
        _ok(gpu_lib, raw.qa_mul_bytes_dev(da.data_ptr(), stride, signed, db.data_ptr(), stride,
                                          signed, dy.data_ptr(), stride, rows, C, 3, -1, mm, ss,
                                          2, qmin, qmax, None))
        np.testing.assert_array_equal(got(), oracle.mul(a32, b32, 3, -1, mm, ss, 2, qmin, qmax))


# (H, W, k, pad): the SPPF window, a 3x3 window, output columns taller than
# one row chunk, a 1x1 image, no padding, and a pad the column walker does
# not take (k5 p1)
POOL_GEOMETRIES = [(9, 11, 5, 2), (9, 11, 3, 1), (40, 3, 5, 2), (1, 1, 3, 1), (7, 8, 5, 0),
                   (9, 11, 5, 1)]


@pytest.mark.parametrize("C,stride,signed", CASES)
@pytest.mark.parametrize("H,W,k,pad", POOL_GEOMETRIES)
def test_maxpool_bytes(gpu_lib, raw, C, stride, signed, H, W, k, pad):
    rng = np.random.default_rng(C + stride + 7 * H + W + k)
    N, st = 2, 1
    qmin = -128 if signed else 0
    x = _vals(rng, (N * H * W, C), signed)
    dx = _dev(x, stride, signed)
    OH, OW = H + 2 * pad - k + 1, W + 2 * pad - k + 1
    dy = torch.zeros(N * OH * OW * stride, dtype=torch.uint8, device="cuda")
    # qmin (the reference's MaxPool padding) and a pad value above some inputs
    for pad_value in (qmin, qmin + 100):
        _ok(gpu_lib, raw.qa_maxpool_bytes_dev(dx.data_ptr(), stride, signed, dy.data_ptr(),
                                              stride, N, H, W, C, k, k, st, st, pad, pad, 1, 1,
                                              OH, OW, pad_value, None))
        xp = np.full((N, H + 2 * pad, W + 2 * pad, C), pad_value, np.int64)
        xp[:, pad:pad + H, pad:pad + W] = x.reshape(N, H, W, C)
        want = np.full((N, OH, OW, C), np.iinfo(np.int64).min)
        for ky in range(k):
            for kx in range(k):
                want = np.maximum(want, xp[:, ky:ky + OH, kx:kx + OW])
        np.testing.assert_array_equal(_host(dy, N * OH * OW, C, stride, signed),
                                      want.reshape(-1, C))
