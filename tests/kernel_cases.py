"""Kernel-level parity cases shared by the oracle and the CUDA-library tests.

Each case runs one ABI entry point on inputs stored in
``tests/golden/kernels.npz`` and returns ``(got, expected, tolerance)``.
Expected values were produced by the reference's own C++ kernels (see
``tests/golden/make_golden.py``); integer results must match bit for bit,
float32 GEMM / conv within the reference's own 1e-4 tolerance
(test_native.py:52, :78-80 in the reference project).
"""

import numpy as np

N_CONV = 8  # CONV_CASES in make_golden.py
N_GEMM = 3
N_EW2 = 12
N_QF = 5


def _conv_args(geom):
    s0, s1, pt, pl, pb, pr, d0, d1, g = (int(v) for v in geom)
    return (s0, s1), (pt, pl, pb, pr), (d0, d1), g


def cases(G):
    """``{name: fn(lib) -> (got, expected, tol)}`` for fixture dict ``G``."""
    out = {}

    for i in range(N_CONV):
        def narrow(lib, i=i):
            return (lib.conv2d_int(G[f"conv{i}_x"], G[f"conv{i}_w"],
                                   *_conv_args(G[f"conv{i}_geom"]), wide=False),
                    G[f"conv{i}_narrow"], 0)

        def wide(lib, i=i):
            return (lib.conv2d_int(G[f"conv{i}_x"], G[f"conv{i}_w"],
                                   *_conv_args(G[f"conv{i}_geom"]), wide=True),
                    G[f"conv{i}_wide"], 0)

        def f32(lib, i=i):
            return (lib.conv2d_f32(G[f"conv{i}_xf"], G[f"conv{i}_wf"],
                                   *_conv_args(G[f"conv{i}_geom"])),
                    G[f"conv{i}_f32"], 1e-4)

        out[f"conv{i}_narrow"], out[f"conv{i}_wide"], out[f"conv{i}_f32"] = narrow, wide, f32

    for kind in ("narrow", "wide"):
        def asym(lib, kind=kind):
            return (lib.conv2d_int(G["convasym_x"], G["convasym_w"],
                                   *_conv_args(G["convasym_geom"]), wide=kind == "wide"),
                    G[f"convasym_{kind}"], 0)

        out[f"convasym_{kind}"] = asym
    out["convtrunc_narrow"] = lambda lib: (
        lib.conv2d_int(G["convtrunc_x"], G["convtrunc_w"], (1, 1), (1, 1, 1, 1),
                       (1, 1), 1, wide=False), G["convtrunc_narrow"], 0)

    for i in range(N_GEMM):
        out[f"gemm{i}_narrow"] = lambda lib, i=i: (
            lib.gemm_int(G[f"gemm{i}_a"], G[f"gemm{i}_b"], False), G[f"gemm{i}_narrow"], 0)
        out[f"gemm{i}_wide"] = lambda lib, i=i: (
            lib.gemm_int(G[f"gemm{i}_a"], G[f"gemm{i}_b"], True), G[f"gemm{i}_wide"], 0)
        out[f"gemm{i}_f32"] = lambda lib, i=i: (
            lib.gemm_f32(G[f"gemm{i}_af"], G[f"gemm{i}_bf"]), G[f"gemm{i}_f32"], 1e-4)
    out["gemmbig_wide"] = lambda lib: (
        lib.gemm_int(G["gemmbig_a"], G["gemmbig_b"], True), G["gemmbig_wide"], 0)

    def rq0(lib):
        o, c, n, zp, lo, hi = (int(v) for v in G["rq0_params"])
        return (lib.requantize(G["rq0_acc"], o, c, n, G["rq0_mult"], G["rq0_shift"],
                               zp, lo, hi, pre_bias=G["rq0_pre"], post_bias=G["rq0_post"]),
                G["rq0_out"], 0)

    out["rq0"] = rq0
    out["rq1"] = lambda lib: (
        lib.requantize(G["rq1_acc"], 2, 3, 20, 1 << 30, 0, 1, -128, 127), G["rq1_out"], 0)
    for qi in range(3):
        def rq2(lib, qi=qi):
            zp, lo, hi = (int(v) for v in G[f"rq2_q{qi}"])
            return (lib.requantize(G["rq2_acc"], 3, 64, 5, G["rq2_mult"], G["rq2_shift"],
                                   zp, lo, hi, pre_bias=G["rq2_pre"],
                                   post_bias=G["rq2_post"]),
                    G[f"rq2_out{qi}"], 0)

        out[f"rq2_{qi}"] = rq2
    out["rq3"] = lambda lib: (
        lib.requantize(G["rq3_acc"], 4, 16, 33, G["rq3_mult"], G["rq3_shift"], -5, -128, 127),
        G["rq3_out"], 0)

    x, y, t = G["ew_x"], G["ew_y"], G["ew_table"]
    out["ew_rescale"] = lambda lib: (lib.rescale(x, 3, 1 << 30, 2, 1, -128, 127),
                                     G["ew_rescale"], 0)
    out["ew_add"] = lambda lib: (
        lib.add(x, y, 0, 1 << 30, 1, 2, 1 << 30, 3, 0, -(2**15), 2**15 - 1, -1),
        G["ew_add"], 0)
    out["ew_mul"] = lambda lib: (lib.mul(x, y, 1, 2, 1 << 30, 10, 0, -128, 127),
                                 G["ew_mul"], 0)
    out["ew_lut"] = lambda lib: (lib.lut(x, t, -50), G["ew_lut"], 0)

    a, b = G["ew2_a"], G["ew2_b"]
    for i in range(N_EW2):
        ma, sa, mb, sb, za, zb, zo, lo, hi, sign = (int(v) for v in G["ew2_params"][i])
        out[f"ew2_rescale{i}"] = lambda lib, za=za, ma=ma, sa=sa, zo=zo, lo=lo, hi=hi, i=i: (
            lib.rescale(a, za, ma, sa, zo, lo, hi), G[f"ew2_rescale{i}"], 0)
        out[f"ew2_add{i}"] = lambda lib, p=(za, ma, sa, zb, mb, sb, zo, lo, hi, sign), i=i: (
            lib.add(a, b, *p), G[f"ew2_add{i}"], 0)
        out[f"ew2_mul{i}"] = lambda lib, p=(za, zb, ma, sa, zo, lo, hi), i=i: (
            lib.mul(a, b, *p), G[f"ew2_mul{i}"], 0)
    out["ew2_lut"] = lambda lib: (lib.lut(a, G["ew2_table"], -32768), G["ew2_lut"], 0)
    out["ew2_lutb"] = lambda lib: (lib.lut(b, G["ew2_table"], -32768), G["ew2_lutb"], 0)

    xf = G["qf_x"]
    for i in range(N_QF):
        sc, zp, lo, hi = G["qf_params"][i]
        out[f"qf_q{i}"] = lambda lib, sc=sc, zp=zp, lo=lo, hi=hi, i=i: (
            lib.quantize_f32(xf, float(sc), int(zp), int(lo), int(hi)), G[f"qf_q{i}"], 0)
        out[f"qf_dq{i}"] = lambda lib, sc=sc, zp=zp, i=i: (
            lib.dequantize_f32(G[f"qf_q{i}"], float(sc), int(zp)), G[f"qf_dq{i}"], 0)
    return out


def check(got, expected, tol):
    """Asserts bit equality (tol == 0) or closeness (float tolerance)."""
    assert got.shape == expected.shape, (got.shape, expected.shape)
    if tol == 0:
        assert got.dtype == expected.dtype, (got.dtype, expected.dtype)
        if got.dtype.kind == "f":
            np.testing.assert_array_equal(got.view(np.uint32), expected.view(np.uint32))
        else:
            np.testing.assert_array_equal(got, expected)
    else:
        np.testing.assert_allclose(got, expected, rtol=tol, atol=tol)
