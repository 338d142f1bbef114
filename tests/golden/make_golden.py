"""Generates the golden fixtures that pin the oracle and the CUDA library.

Run in the development container, where the reference project is importable:

    python tests/golden/make_golden.py [--ref <reference checkout>] [--graphs]

(--ref defaults to $QA_REFERENCE_ROOT, else a directory named `reference`
beside this repository.)

Every expected value below is produced by the REFERENCE itself: its Python
package (quantization/*) imported read-only with an import stub for the
absent `onnx` package, driving its own C++ kernels compiled from its own
source by oracle/Makefile (`oracle/_ref/libqa_kernels_ref.so`, loaded through
the reference's QA_LIB switch).  Nothing here reads the oracle or the CUDA
library, so the fixtures are an independent pin for both.

Outputs (all small; large tensors are stored as SHA-256 digests):
  kernels.npz        kernel-level cases mirroring the reference's unit tests
                     plus edge cases of the fixed-point multiply
  host_math.json     quantize_multiplier / calculate_scale_zp known answers
  configs.json       digests of the cfg0 / cfg1 full-size outputs
  graphs/*.npz|json  (with --graphs) quantized-graph fixtures
"""

import argparse
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def _setup_reference(ref_root):
    sys.path.insert(0, str(HERE / "_onnx_stub"))
    sys.path.insert(0, str(ref_root))
    sys.path.insert(0, str(REPO))
    lib = REPO / "oracle" / "_ref" / "libqa_kernels_ref.so"
    if not lib.exists():
        raise SystemExit("build the reference library first: make -C oracle ref")
    os.environ["QA_LIB"] = str(lib)
    from quantization import native  # noqa: E402

    if not native.available() or native._lib.qa_has_openmp() != 1:
        raise SystemExit(f"reference kernels not loaded: {native.load_error()}")
    return native


def digest(a):
    """SHA-256 of an array's dtype, shape and C-order bytes."""
    a = np.ascontiguousarray(a)
    h = hashlib.sha256()
    h.update(str(a.dtype).encode())
    h.update(str(a.shape).encode())
    h.update(a.tobytes())
    return h.hexdigest()


# Conv geometries of the reference's kernel tests (test_native.py:8-15):
# N, C, H, W, Cout, K, stride, pad, dilation, groups.
CONV_CASES = [
    (2, 6, 9, 11, 8, 3, 1, 1, 1, 1),
    (1, 8, 16, 16, 8, 3, 2, 1, 1, 8),
    (2, 4, 10, 10, 6, 1, 1, 0, 1, 2),
    (1, 3, 12, 12, 4, 3, 1, 2, 2, 1),
    (3, 5, 7, 7, 5, 5, 1, 0, 1, 1),
    # extra: tensor-core friendly shapes (channel counts multiple of 16)
    (2, 32, 14, 14, 48, 3, 1, 1, 1, 1),
    (1, 64, 9, 9, 32, 3, 2, 1, 1, 1),
    (2, 16, 8, 8, 16, 1, 1, 0, 1, 1),
]


def kernel_cases(native):
    out = {}
    # --- integer conv, both widths (test_native.py:30-40) -------------------
    for ci, case in enumerate(CONV_CASES):
        n, c, h, w_, co, k, s, p, d, g = case
        rng = np.random.default_rng(100 + ci)
        x = rng.integers(-255, 256, (n, c, h, w_)).astype(np.int32)
        w = rng.integers(-128, 128, (co, c // g, k, k)).astype(np.int32)
        args = ((s, s), (p, p, p, p), (d, d), g)
        out[f"conv{ci}_x"] = x
        out[f"conv{ci}_w"] = w
        out[f"conv{ci}_geom"] = np.array([s, s, p, p, p, p, d, d, g], np.int64)
        out[f"conv{ci}_narrow"] = native.conv2d_int(x, w, *args, wide=False)
        out[f"conv{ci}_wide"] = native.conv2d_int(x, w, *args, wide=True)
        xf = rng.standard_normal(x.shape).astype(np.float32)
        wf = rng.standard_normal(w.shape).astype(np.float32)
        out[f"conv{ci}_xf"] = xf
        out[f"conv{ci}_wf"] = wf
        out[f"conv{ci}_f32"] = native.conv2d_f32(xf, wf, *args)
    # asymmetric padding and strides (test_native.py:55-61)
    rng = np.random.default_rng(3)
    x = rng.integers(-9, 9, (1, 2, 6, 6)).astype(np.int32)
    w = rng.integers(-9, 9, (3, 2, 3, 3)).astype(np.int32)
    out["convasym_x"], out["convasym_w"] = x, w
    out["convasym_geom"] = np.array([1, 2, 0, 2, 1, 0, 1, 1, 1], np.int64)
    out["convasym_wide"] = native.conv2d_int(
        x, w, (1, 2), (0, 2, 1, 0), (1, 1), 1, wide=True
    )
    out["convasym_narrow"] = native.conv2d_int(
        x, w, (1, 2), (0, 2, 1, 0), (1, 1), 1, wide=False
    )
    # narrow path with inputs outside int16: the reference casts to int16
    rng = np.random.default_rng(11)
    x = rng.integers(-(2**20), 2**20, (1, 4, 5, 5)).astype(np.int32)
    w = rng.integers(-300, 300, (2, 4, 3, 3)).astype(np.int32)
    out["convtrunc_x"], out["convtrunc_w"] = x, w
    out["convtrunc_narrow"] = native.conv2d_int(
        x, w, (1, 1), (1, 1, 1, 1), (1, 1), 1, wide=False
    )
    # --- integer GEMM (test_native.py:64-71) + tile-crossing shapes ---------
    for gi, (m, k, n) in enumerate([(7, 37, 530), (130, 200, 96), (1, 5, 3)]):
        rng = np.random.default_rng(4 + gi)
        a = rng.integers(-255, 256, (m, k)).astype(np.int32)
        b = rng.integers(-128, 128, (k, n)).astype(np.int32)
        out[f"gemm{gi}_a"], out[f"gemm{gi}_b"] = a, b
        out[f"gemm{gi}_narrow"] = native.gemm_int(a, b, False)
        out[f"gemm{gi}_wide"] = native.gemm_int(a, b, True)
        af = rng.standard_normal((m, k)).astype(np.float32)
        bf = rng.standard_normal((k, n)).astype(np.float32)
        out[f"gemm{gi}_af"], out[f"gemm{gi}_bf"] = af, bf
        out[f"gemm{gi}_f32"] = native.gemm_f32(af, bf)
    # wide GEMM with full-range int32 operands
    rng = np.random.default_rng(9)
    a = rng.integers(-(2**31), 2**31, (9, 70)).astype(np.int32)
    b = rng.integers(-(2**31), 2**31, (70, 33)).astype(np.int32)
    out["gemmbig_a"], out["gemmbig_b"] = a, b
    out["gemmbig_wide"] = native.gemm_int(a, b, True)
    # --- requantize (test_native.py:89-110) + fixed-point edge cases -------
    rng = np.random.default_rng(6)
    acc = rng.integers(-(2**40), 2**40, (2, 5, 7)).astype(np.int64)
    mult = rng.integers(-(2**31) + 1, 2**31, 5)
    shift = rng.integers(-3, 25, 5)
    pre, post = rng.integers(-50, 50, 5), rng.integers(-50, 50, 5)
    out["rq0_acc"], out["rq0_mult"], out["rq0_shift"] = acc, mult, shift
    out["rq0_pre"], out["rq0_post"] = pre, post
    out["rq0_params"] = np.array([2, 5, 7, 3, -32768, 32767], np.int64)
    out["rq0_out"] = native.requantize(
        acc, 2, 5, 7, mult, shift, 3, -32768, 32767, pre_bias=pre, post_bias=post
    )
    acc = np.arange(-60, 60, dtype=np.int32).reshape(2, 3, 20)
    out["rq1_acc"] = acc
    out["rq1_out"] = native.requantize(acc, 2, 3, 20, 1 << 30, 0, 1, -128, 127)
    # edge cases: every branch of mbqm (ts > 64, ts capped at 120, ts <= 0,
    # ts capped at -60), negative multipliers, huge accumulators, wide ranges
    rng = np.random.default_rng(12)
    C = 64
    shift = np.concatenate(
        [
            np.arange(-100, -28),  # ts <= 3 incl. left shifts and the -60 cap
            np.arange(-3, 40),
            np.array([60, 80, 89, 90, 100, 150]),  # ts > 64, cap at 120
        ]
    )[:C].astype(np.int64)
    shift = np.resize(shift, C)
    rng.shuffle(shift)
    mult = rng.integers(-(2**31) + 1, 2**31, C).astype(np.int64)
    mult[:4] = [0, 1, -1, 2**31 - 1]
    acc = rng.integers(-(2**62), 2**62, (3, C, 5)).astype(np.int64)
    acc[0, :, 0] = 2**63 - 1
    acc[1, :, 0] = -(2**63) + 60  # pre_bias stays inside int64
    pre = rng.integers(-50, 50, C).astype(np.int64)
    post = rng.integers(-(2**40), 2**40, C).astype(np.int64)
    out["rq2_acc"], out["rq2_mult"], out["rq2_shift"] = acc, mult, shift
    out["rq2_pre"], out["rq2_post"] = pre, post
    for qi, (zp, lo, hi) in enumerate(
        [(7, -(2**31), 2**31 - 1), (-3, -128, 127), (0, -(2**62), 2**62)]
    ):
        out[f"rq2_out{qi}"] = native.requantize(
            acc, 3, C, 5, mult, shift, zp, lo, hi, pre_bias=pre, post_bias=post
        )
        out[f"rq2_q{qi}"] = np.array([zp, lo, hi], np.int64)
    # int32 accumulators, full range, per-channel params, no biases
    acc = rng.integers(-(2**31), 2**31, (4, 16, 33)).astype(np.int32)
    mult = rng.integers(2**30, 2**31, 16).astype(np.int64)
    shift = rng.integers(-2, 20, 16).astype(np.int64)
    out["rq3_acc"], out["rq3_mult"], out["rq3_shift"] = acc, mult, shift
    out["rq3_out"] = native.requantize(acc, 4, 16, 33, mult, shift, -5, -128, 127)
    # --- element-wise kernels (test_native.py:113-139) ----------------------
    rng = np.random.default_rng(7)
    x = rng.integers(-1000, 1000, 1000).astype(np.int32)
    y = x[::-1].copy()
    table = np.arange(100, dtype=np.int32)
    out["ew_x"], out["ew_y"], out["ew_table"] = x, y, table
    out["ew_rescale"] = native.rescale(x, 3, 1 << 30, 2, 1, -128, 127)
    out["ew_add"] = native.add(
        x, y, 0, 1 << 30, 1, 2, 1 << 30, 3, 0, -(2**15), 2**15 - 1, -1
    )
    out["ew_mul"] = native.mul(x, y, 1, 2, 1 << 30, 10, 0, -128, 127)
    out["ew_lut"] = native.lut(x, table, -50)
    # larger random element-wise cases with multiplier/shift sweeps
    rng = np.random.default_rng(13)
    n = 4099
    a = rng.integers(-(2**31), 2**31, n).astype(np.int32)
    b = rng.integers(-(2**15), 2**15, n).astype(np.int32)
    out["ew2_a"], out["ew2_b"] = a, b
    params = []
    for i in range(12):
        ma, mb = (int(v) for v in rng.integers(-(2**31) + 1, 2**31, 2))
        sa, sb = (int(v) for v in rng.integers(-40, 70, 2))
        za, zb, zo = (int(v) for v in rng.integers(-300, 300, 3))
        lo, hi = [(-128, 127), (0, 255), (-(2**31), 2**31 - 1)][i % 3]
        sign = 1 if i % 2 else -1
        params.append([ma, sa, mb, sb, za, zb, zo, lo, hi, sign])
        out[f"ew2_rescale{i}"] = native.rescale(a, za, ma, sa, zo, lo, hi)
        out[f"ew2_add{i}"] = native.add(a, b, za, ma, sa, zb, mb, sb, zo, lo, hi, sign)
        out[f"ew2_mul{i}"] = native.mul(a, b, za, zb, ma, sa, zo, lo, hi)
    out["ew2_params"] = np.array(params, np.int64)
    tbl = rng.integers(-(2**15), 2**15, 65536).astype(np.int32)
    out["ew2_table"] = tbl
    out["ew2_lut"] = native.lut(a, tbl, -32768)
    out["ew2_lutb"] = native.lut(b, tbl, -32768)
    # --- float <-> integer (utils.py:97-124 fast path) ---------------------
    rng = np.random.default_rng(14)
    xf = np.concatenate(
        [
            rng.uniform(-3, 5, 5000).astype(np.float32),
            np.array([0.5, 1.5, 2.5, -0.5, -1.5, 1e6, -1e6, np.inf, -np.inf,
                      0.0, -0.0, 1e-30], np.float32),
            (np.arange(-300, 300).astype(np.float32) + 0.5) * np.float32(0.25),
        ]
    )
    out["qf_x"] = xf
    qparams = [(1.0, 0, -128, 127), (0.25, 0, -128, 127), (0.0314, 17, 0, 255),
               (3.0 / 32767.0, 0, -32768, 32767), (1e-3, -7, -(2**31), 2**31 - 1)]
    out["qf_params"] = np.array(qparams, np.float64)
    for i, (sc, zp, lo, hi) in enumerate(qparams):
        q = native.quantize_f32(xf, sc, zp, lo, hi)
        out[f"qf_q{i}"] = q
        out[f"qf_dq{i}"] = native.dequantize_f32(q, sc, zp)
    return out


def host_math_cases():
    """Known answers of the reference's host parameter derivation."""
    from quantization.utils import calculate_scale_zp, quantize_multiplier

    rng = np.random.default_rng(15)
    reals = [1e-5, 0.0123, 0.5, 1.0, 3.7, 250.0, -0.3, 0.0, 2.0**-40, 0.9999999999]
    reals += [float(v) for v in rng.uniform(1e-6, 10, 40)]
    mult = [list(quantize_multiplier(r)) for r in reals]
    ranges = [(-10.0, 10.0), (-2.0, 8.0), (2.0, 10.0), (-100.0, 50.0), (0.0, 0.0),
              (-3.1, 0.7), (-0.278, 6.5)]
    types = ["int8", "uint8", "int16", "uint16", "int9"]
    scz = []
    for lo, hi in ranges:
        for t in types:
            scz.append([lo, hi, t, list(calculate_scale_zp(lo, hi, t))])
    return {"multipliers": [[r, m] for r, m in zip(reals, mult)], "scale_zp": scz}


def config_digests(native):
    from quantanything_b200 import configs
    from quantization.utils import dequantize, quantize

    res = {}
    c0 = configs.linear_cfg0()
    acc = native.gemm_int(c0.a - c0.a_zp, np.ascontiguousarray(c0.w.T), False)
    out0 = native.requantize(
        acc, acc.shape[0], acc.shape[1], 1, c0.mult, c0.shift, c0.out_zp,
        c0.qmin, c0.qmax, pre_bias=c0.bias,
    )
    res["cfg0"] = {"acc": digest(acc), "out": digest(out0),
                   "out_head": out0[0, :16].tolist()}
    c1 = configs.conv_cfg1()
    acc = native.conv2d_int(c1.x - c1.x_zp, c1.w, (1, 1), (1, 1, 1, 1), (1, 1), 1,
                            wide=False)
    n, co, oh, ow = acc.shape
    mid = native.requantize(acc, n, co, oh * ow, c1.mult, c1.shift, c1.mid_zp,
                            c1.qmin, c1.qmax, pre_bias=c1.bias)
    # SiLU table exactly as ActivationQuantize.prepare builds it
    q_in = np.arange(c1.qmin, c1.qmax + 1, dtype=np.int64)
    xin = dequantize(q_in.astype(np.int32), c1.mid_scale, c1.mid_zp)
    sig = (1.0 / (1.0 + np.exp(-xin.astype(np.float64)))).astype(np.float32)
    y = np.multiply(xin, sig)
    table = quantize(y, c1.out_scale, c1.out_zp, c1.qmin, c1.qmax).astype(np.int32)
    out1 = native.lut(mid, table, c1.qmin)
    res["cfg1"] = {"acc": digest(acc), "mid": digest(mid), "out": digest(out1),
                   "table": table.tolist(), "out_head": out1[0, 0, 0, :16].tolist()}
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("QA_REFERENCE_ROOT",
                                                  str(REPO.parent / "reference")))
    ap.add_argument("--graphs", action="store_true")
    ap.add_argument("--only", nargs="*", help="graph fixtures to (re)write; nothing else")
    args = ap.parse_args()
    native = _setup_reference(Path(args.ref))
    if not args.only:
        np.savez_compressed(HERE / "kernels.npz", **kernel_cases(native))
        (HERE / "host_math.json").write_text(json.dumps(host_math_cases(), indent=1))
        (HERE / "configs.json").write_text(json.dumps(config_digests(native), indent=1))
    if args.graphs or args.only:
        from tests.golden import graph_fixtures  # noqa: E402

        graph_fixtures.generate(HERE / "graphs", args.only)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
