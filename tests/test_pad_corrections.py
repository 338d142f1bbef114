"""Border correction tables of the fused conv's TMA gather (host side).

With a nonzero input zero point the TMA im2col gather reads out-of-image
taps as 0 where the reference pads with the zero point (its integer conv
centres every tap, so a padded tap contributes nothing); the epilogue adds
x_zp * (weights over the out-of-image taps) per border class.  Checked here
against a direct enumeration of every output pixel's taps.
"""
import numpy as np
import pytest

from quantanything_b200.resident import pad_corrections


def _brute(wt, zp, H, W, KH, KW, SH, SW, PH, PW, DH, DW, OH, OW):
    out = np.zeros((OH, OW, wt.shape[0]), np.int64)
    for oy in range(OH):
        for ox in range(OW):
            for ky in range(KH):
                for kx in range(KW):
                    iy, ix = oy * SH - PH + ky * DH, ox * SW - PW + kx * DW
                    if not (0 <= iy < H and 0 <= ix < W):
                        out[oy, ox] += zp * wt[:, ky, kx, :].sum(axis=1)
    return out


@pytest.mark.parametrize("geo", [
    dict(H=9, W=7, KH=3, KW=3, SH=1, SW=1, PH=1, PW=1, DH=1, DW=1),
    dict(H=10, W=10, KH=3, KW=3, SH=2, SW=2, PH=1, PW=1, DH=1, DW=1),
    dict(H=8, W=11, KH=3, KW=3, SH=1, SW=1, PH=2, PW=2, DH=2, DW=2),
    dict(H=6, W=6, KH=1, KW=3, SH=1, SW=1, PH=0, PW=1, DH=1, DW=1),
])
@pytest.mark.parametrize("zp", [7, -5])
def test_pad_corrections_match_enumeration(geo, zp):
    rng = np.random.default_rng(1)
    OH = (geo["H"] + 2 * geo["PH"] - geo["DH"] * (geo["KH"] - 1) - 1) // geo["SH"] + 1
    OW = (geo["W"] + 2 * geo["PW"] - geo["DW"] * (geo["KW"] - 1) - 1) // geo["SW"] + 1
    wt = rng.integers(-127, 128, (5, geo["KH"], geo["KW"], 16))
    pc = pad_corrections(wt, zp, OH=OH, OW=OW, **geo)
    assert pc is not None
    corr, rcls, ccls, ncol = pc
    got = corr[(rcls[:, None] * ncol + ccls[None, :])]
    np.testing.assert_array_equal(got, _brute(wt, zp, OH=OH, OW=OW, **geo))
    assert corr[0].tolist() == [0] * 5  # class 0: interior pixels


def test_no_tables_without_zero_point_or_padding():
    wt = np.ones((2, 3, 3, 16), np.int64)
    geo = dict(H=8, W=8, KH=3, KW=3, SH=1, SW=1, PH=1, PW=1, DH=1, DW=1, OH=8, OW=8)
    assert pad_corrections(wt, 0, **geo) is None
    geo.update(PH=0, PW=0, OH=6, OW=6)
    assert pad_corrections(wt, 3, **geo) is None
