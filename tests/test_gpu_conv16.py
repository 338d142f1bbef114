"""qa_conv16_fused_dev (the int16 resident contraction) vs the C oracle.

Every conv geometry of the reference's own kernel tests (the golden
fixture's CONV_CASES: plain, depthwise strided, grouped pointwise, dilated,
big kernel without padding, wide channels, strided, pointwise, asymmetric
padding) runs on random int16 operands through the fused 16-bit kernel --
dense layers on the byte-split tensor cores, grouped ones on CUDA cores --
and must equal, bit for bit, the reference's wide route on the oracle:
int64 convolution of the centred input, requantize (128-bit mbqm), the
activation table, the residual Add and the rescaled Concat copy
(qa_kernels.cpp:281-284, 207-228, 307-358).
"""
import ctypes

import numpy as np
import pytest
import torch

from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu
G = dict(np.load(GOLDEN / "kernels.npz"))
GEOMS = [f"conv{i}" for i in range(8)] + ["convasym"]


def _ru(v, m):
    return (v + m - 1) // m * m


def _to_planes(x_nhwc, pix_stride, fill):
    """int16 values [N,H,W,C] -> device bytes (low plane, then high plane)."""
    N, H, W, C = x_nhwc.shape
    rows = N * H * W
    plane = _ru(rows * pix_stride, 256)
    v = np.full((rows, pix_stride), fill, np.int64)
    v[:, :C] = x_nhwc.reshape(rows, C)
    buf = np.zeros(2 * plane, np.uint8)
    buf[:rows * pix_stride] = (v & 0xFF).astype(np.uint8).ravel()
    buf[plane:plane + rows * pix_stride] = ((v >> 8) & 0xFF).astype(np.uint8).ravel()
    return torch.from_numpy(buf).cuda(), plane


def _from_planes(buf, plane, N, H, W, C, pix_stride):
    b = buf.cpu().numpy()
    rows = N * H * W
    lo = b[:rows * pix_stride].reshape(rows, pix_stride)[:, :C].astype(np.int64)
    hi = b[plane:plane + rows * pix_stride].reshape(rows, pix_stride)[:, :C].view(np.int8)
    return (lo + 256 * hi.astype(np.int64)).reshape(N, H, W, C)


def _run(gpu_lib, oracle, name, epi, x_zp, seed, block_n=None):
    from quantanything_b200 import native
    from quantanything_b200.resident import device_api
    from quantanything_b200.resident16 import FusedConv16Desc, device_api16

    device_api(gpu_lib)
    raw = device_api16(gpu_lib)
    rng = np.random.default_rng(seed)
    s0, s1, pt, pl, pb, pr, d0, d1, groups = (int(v) for v in G[f"{name}_geom"])
    N, C, H, W = G[f"{name}_x"].shape
    Cout, Cg, KH, KW = G[f"{name}_w"].shape
    xr = rng.integers(-32768, 32768, (N, C, H, W))
    w = rng.integers(-32767, 32768, (Cout, Cg, KH, KW))
    g = native.conv_geometry((N, C, H, W), w.shape, (s0, s1), (pt, pl, pb, pr), (d0, d1),
                             groups)
    OH, OW = g[13], g[14]
    bias = rng.integers(-(2**40), 2**40, Cout)
    mult = rng.integers(2**30, 2**31, Cout)
    shift = rng.integers(18, 27, Cout)
    mult[0], shift[1] = -mult[0], -2          # exact 128-bit fallback channels
    qmin, qmax, zp = -32768, 32767, int(rng.integers(-50, 50))

    # ---- oracle: the reference's wide route on the centred input
    acc = oracle.conv2d_int((xr - x_zp).astype(np.int32), w.astype(np.int32), (s0, s1),
                            (pt, pl, pb, pr), (d0, d1), groups, wide=True)
    want = oracle.requantize(acc, N, Cout, OH * OW, mult, shift, zp, qmin, qmax,
                             pre_bias=bias)
    table = rng.integers(-32768, 32768, 65536).astype(np.int32)
    if epi in ("lut", "lut16", "res"):
        want = oracle.lut(want, table, -32768)
    res = rng.integers(-32768, 32768, (N, Cout, OH, OW))
    ap = dict(za=int(rng.integers(-9, 9)), ma=int(rng.integers(2**30, 2**31)), sa=1,
              zb=int(rng.integers(-9, 9)), mb=int(rng.integers(2**30, 2**31)), sb=0, zo=3)
    rp = dict(zin=5, m=int(rng.integers(2**30, 2**31)), s=1, zout=-7)
    want2 = None
    if epi == "res":
        want = oracle.add(res.astype(np.int32), want, ap["za"], ap["ma"], ap["sa"], ap["zb"],
                          ap["mb"], ap["sb"], ap["zo"], qmin, qmax)
        want2 = oracle.rescale(want, rp["zin"], rp["m"], rp["s"], rp["zout"], qmin, qmax)

    # ---- the fused 16-bit kernel
    ct = C if groups > 1 or C % 16 == 0 else _ru(C, 4)
    if groups > 1:
        ct = Cg
    xs = C if C % 16 == 0 else _ru(C, 16)
    xdev, xplane = _to_planes(np.transpose(xr, (0, 2, 3, 1)), xs, x_zp)
    bn = 0 if groups > 1 else (16 if Cout <= 16 else 32 if Cout <= 32 else 64)
    if block_n and groups == 1:
        bn = block_n
    rows = _ru(Cout, bn or 16)
    K = KH * KW * ct
    kp = _ru(K, 16)
    wt = np.zeros((Cout, KH, KW, ct), np.int64)
    wt[..., :Cg] = np.transpose(w, (0, 2, 3, 1))
    packed = np.zeros((rows, kp), np.int64)
    packed[:Cout, :K] = wt.reshape(Cout, K)
    wdev = torch.from_numpy(np.concatenate([(packed & 0xFF), (packed >> 8) & 0xFF])
                            .astype(np.uint8)).cuda()
    bdev = torch.from_numpy(bias - x_zp * wt.reshape(Cout, -1).sum(axis=1)).cuda()
    mdev, sdev = torch.from_numpy(mult).cuda(), torch.from_numpy(shift).cuda()
    os_ = Cout if Cout % 16 == 0 else _ru(Cout, 16)
    odev, oplane = _to_planes(np.zeros((N, OH, OW, Cout), np.int64), os_, 0)
    d = FusedConv16Desc()
    b = d.base
    b.x, b.x_pix_stride, b.x_signed, b.x_zp = xdev.data_ptr(), xs, 1, x_zp
    b.N, b.H, b.W, b.C = N, H, W, ct
    b.KH, b.KW, b.SH, b.SW, b.PH, b.PW, b.DH, b.DW = KH, KW, s0, s1, pt, pl, d0, d1
    b.OH, b.OW, b.Cout, b.groups = OH, OW, Cout, groups
    b.w, b.w_rows, b.w_kp = wdev.data_ptr(), rows, kp
    b.bias, b.mult, b.shift = bdev.data_ptr(), mdev.data_ptr(), sdev.data_ptr()
    b.zp, b.qmin, b.qmax = zp, qmin, qmax
    b.out, b.out_pix_stride, b.block_n = odev.data_ptr(), os_, bn
    d.x_plane, d.out_plane = xplane, oplane
    keep = []
    if epi in ("lut", "lut16", "res"):
        tdev = torch.from_numpy(table).cuda()
        keep.append(tdev)
        b.lut, b.lut_offset, b.lut_len = tdev.data_ptr(), -32768, 65536
        if epi in ("lut16", "res"):
            t16 = tdev.to(torch.int16)
            keep.append(t16)
            d.lut16 = t16.data_ptr()
    if epi == "res":
        rdev, rplane = _to_planes(np.transpose(res, (0, 2, 3, 1)), os_, 0)
        o2dev, o2plane = _to_planes(np.zeros((N, OH, OW, Cout), np.int64), os_, 0)
        keep += [rdev, o2dev]
        b.res, b.res_pix_stride, b.res_signed = rdev.data_ptr(), os_, 1
        b.za, b.ma, b.sa, b.zb, b.mb, b.sb = (ap[k] for k in ("za", "ma", "sa", "zb", "mb",
                                                             "sb"))
        b.sign, b.add_zo, b.add_qmin, b.add_qmax = 1, ap["zo"], qmin, qmax
        b.out2, b.out2_pix_stride = o2dev.data_ptr(), os_
        b.r_identity, b.r_zp_in, b.r_m, b.r_s = 0, rp["zin"], rp["m"], rp["s"]
        b.r_zp_out, b.r_qmin, b.r_qmax = rp["zout"], qmin, qmax
        d.res_plane, d.out2_plane = rplane, o2plane
    rc = raw.qa_conv16_fused_dev(ctypes.byref(d), None)
    assert rc == 0, gpu_lib.raw.qa_last_error().decode()
    torch.cuda.synchronize()
    assert raw.qa_device_status_dev(None) == 0
    got = np.transpose(_from_planes(odev, oplane, N, OH, OW, Cout, os_), (0, 3, 1, 2))
    np.testing.assert_array_equal(got, want)
    if want2 is not None:
        got2 = np.transpose(_from_planes(o2dev, o2plane, N, OH, OW, Cout, os_), (0, 3, 1, 2))
        np.testing.assert_array_equal(got2, want2)


EPIS = [("plain", 0), ("lut", 37), ("lut16", 0), ("res", -5)]


@pytest.mark.parametrize("name", GEOMS)
@pytest.mark.parametrize("epi,x_zp", EPIS)
def test_conv16_matches_wide_route(gpu_lib, oracle, name, epi, x_zp):
    seed = 100 * GEOMS.index(name) + EPIS.index((epi, x_zp))
    _run(gpu_lib, oracle, name, epi, x_zp, seed=seed)


@pytest.mark.parametrize("name", [g for g in GEOMS if int(G[f"{g}_geom"][8]) == 1])
@pytest.mark.parametrize("epi,x_zp", [("lut", 11), ("res", 0)])
def test_conv16_wide_column_tile(gpu_lib, oracle, name, epi, x_zp):
    """128-column tiles: one TMEM accumulator set, both epilogue warpgroups
    on every tile (half the columns each), the table in global memory."""
    _run(gpu_lib, oracle, name, epi, x_zp, seed=7 + GEOMS.index(name), block_n=128)
