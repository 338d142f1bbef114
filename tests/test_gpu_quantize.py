"""Graph-input quantization on the B200 vs the reference's qa_quantize_f32.

The device kernels round x / scale through a float product with 1/scale and
fall back to the double division near half-integers (ties included), for
NaN / inf and for scales they cannot invert.  These inputs sit on and
around every half-integer of the output range, so a wrong fallback bound
shows up as a changed byte.
"""
import ctypes

import numpy as np
import pytest
import torch

from quantanything_b200.resident import device_api

pytestmark = pytest.mark.gpu

# (scale, zp, qmin, qmax): the golden YOLO input, an asymmetric int8 and a
# uint8 mapping, and scales too small / too large for the float path
CASES = [
    (0.023622047244094488, 0, -128, 127),
    (0.1, -5, -128, 127),
    (0.0078125, 128, 0, 255),
    (1e-35, 3, -128, 127),
    (3e35, 0, -128, 127),
]


def _adversarial(scale, rng):
    k = np.arange(-300, 301, dtype=np.float64)
    ties = ((k + 0.5) * scale).astype(np.float32)
    near = np.concatenate([ties, np.nextafter(ties, np.float32(np.inf)),
                           np.nextafter(ties, np.float32(-np.inf)),
                           np.nextafter(np.nextafter(ties, np.float32(np.inf)), np.float32(np.inf))])
    ints = (k * scale).astype(np.float32)
    special = np.array([np.nan, np.inf, -np.inf, 1e30, -1e30, 3.4e38, -3.4e38, 1e-40, -1e-40,
                        0.0, -0.0, 1e-30], np.float32)
    rand = rng.standard_normal(4096).astype(np.float32) * 3
    return np.concatenate([near, ints, special, rand])


@pytest.mark.parametrize("scale,zp,qmin,qmax", CASES)
def test_quantize_to_nhwc_matches_reference(gpu_lib, oracle, scale, zp, qmin, qmax):
    vals = _adversarial(scale, np.random.default_rng(5))
    C, H = 3, 8
    W = -(-vals.size // (C * H))
    W += (-W) % 4  # H * W a multiple of 4: the 4-pixel kernel
    x = np.zeros(C * H * W, np.float32)
    x[:vals.size] = vals
    x = x.reshape(1, C, H, W)
    want = oracle.quantize_f32(x, scale, zp, qmin, qmax)  # int32, NCHW
    raw = device_api(gpu_lib)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(H * W * 4, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    rc = raw.qa_quantize_to_nhwc_dev(xd.data_ptr(), yd.data_ptr(), 1, C, H, W, 4, float(scale),
                                     zp, qmin, qmax, ctypes.c_void_p(st))
    assert rc == 0
    torch.cuda.synchronize()
    got = yd.cpu().numpy().reshape(H * W, 4)
    want_b = (want.reshape(C, H * W).T.astype(np.int64) & 0xFF).astype(np.uint8)
    np.testing.assert_array_equal(got[:, :C], want_b)
    assert (got[:, C] == (zp & 0xFF)).all()


@pytest.mark.parametrize("P,H,W", [(16, 32, 48), (8, 16, 8), (4, 12, 20)])
def test_patch_rows_are_the_nhwc_bytes_in_im2col_order(gpu_lib, oracle, P, H, W):
    """qa_quantize_to_patch_rows_dev: the same bytes as the NHWC quantizer
    (pinned to the reference above), rearranged into the im2col rows of a
    P x P, stride-P conv: row (n, py, px), pixel (ky, kx) at (ky * P + kx) * 4."""
    rng = np.random.default_rng(P)
    N, C, scale, zp = 2, 3, 0.02, 7
    x = (rng.standard_normal((N, C, H, W)) * 2).astype(np.float32)
    raw = device_api(gpu_lib)
    xd = torch.from_numpy(x).cuda()
    nhwc = torch.empty(N * H * W * 4, dtype=torch.uint8, device="cuda")
    rows = torch.empty_like(nhwc)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert raw.qa_quantize_to_nhwc_dev(xd.data_ptr(), nhwc.data_ptr(), N, C, H, W, 4, scale, zp,
                                       -128, 127, st) == 0
    assert raw.qa_quantize_to_patch_rows_dev(xd.data_ptr(), rows.data_ptr(), N, C, H, W, P,
                                             scale, zp, -128, 127, st) == 0
    torch.cuda.synchronize()
    a = nhwc.cpu().numpy().reshape(N, H // P, P, W // P, P, 4).transpose(0, 1, 3, 2, 4, 5)
    np.testing.assert_array_equal(rows.cpu().numpy().reshape(a.shape), a)
    want = oracle.quantize_f32(x, scale, zp, -128, 127)
    assert (nhwc.cpu().numpy().reshape(N, H, W, 4)[..., :C].view(np.int8)
            == want.transpose(0, 2, 3, 1)).all()
