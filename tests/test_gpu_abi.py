"""Parity of the CUDA library's reference ABI (host pointers) on a B200.

Every golden case of the reference's kernel tests is replayed through the
CUDA library (bit-exact for integers, the reference's 1e-4 for float32), and
larger seeded shapes that cross tile, K-block and pipeline boundaries are
checked against the C oracle on the same inputs.
"""
import json

import numpy as np
import pytest

from tests import kernel_cases
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

_G = dict(np.load(GOLDEN / "kernels.npz"))
_CASES = kernel_cases.cases(_G)


@pytest.mark.parametrize("name", sorted(_CASES))
def test_golden_case(gpu_lib, name):
    got, expected, tol = _CASES[name](gpu_lib)
    kernel_cases.check(got, expected, tol)


GEMM_SHAPES = [(300, 1000, 200), (128, 128, 64), (129, 1, 65), (64, 4100, 3), (517, 96, 77)]


@pytest.mark.parametrize("m,k,n", GEMM_SHAPES)
def test_gemm_narrow_vs_oracle(gpu_lib, oracle, m, k, n):
    rng = np.random.default_rng(m * 7 + k)
    a = rng.integers(-(2**15), 2**15, (m, k)).astype(np.int16)
    b = rng.integers(-(2**15), 2**15, (k, n)).astype(np.int16)
    np.testing.assert_array_equal(gpu_lib.gemm_int(a, b, False), oracle.gemm_int(a, b, False))


@pytest.mark.parametrize("m,k,n", GEMM_SHAPES[:3])
def test_gemm_wide_vs_oracle(gpu_lib, oracle, m, k, n):
    rng = np.random.default_rng(m + k * 3)
    a = rng.integers(-(2**31), 2**31, (m, k)).astype(np.int32)
    b = rng.integers(-(2**31), 2**31, (k, n)).astype(np.int32)
    np.testing.assert_array_equal(gpu_lib.gemm_int(a, b, True), oracle.gemm_int(a, b, True))


CONV_SHAPES = [
    # N, C, H, W, Cout, K, stride, pad, dilation, groups
    (2, 64, 20, 18, 96, 3, 1, 1, 1, 1),
    (1, 32, 17, 17, 64, 3, 2, 1, 1, 2),
    (3, 16, 9, 9, 130, 1, 1, 0, 1, 1),
    (1, 48, 11, 13, 16, 5, 1, 2, 2, 1),
    (2, 3, 32, 32, 16, 3, 2, 1, 1, 1),
]


@pytest.mark.parametrize("case", CONV_SHAPES)
@pytest.mark.parametrize("wide", [False, True])
def test_conv_vs_oracle(gpu_lib, oracle, case, wide):
    n, c, h, w_, co, k, s, p, d, g = case
    rng = np.random.default_rng(sum(case))
    x = rng.integers(-(2**15), 2**15, (n, c, h, w_)).astype(np.int32)
    w = rng.integers(-(2**15), 2**15, (co, c // g, k, k)).astype(np.int32)
    args = ((s, s), (p, p, p, p), (d, d), g)
    np.testing.assert_array_equal(gpu_lib.conv2d_int(x, w, *args, wide=wide),
                                  oracle.conv2d_int(x, w, *args, wide=wide))


def test_requantize_large_vs_oracle(gpu_lib, oracle):
    rng = np.random.default_rng(21)
    acc = rng.integers(-(2**31), 2**31, (8, 96, 1001)).astype(np.int32)
    mult = rng.integers(-(2**31) + 1, 2**31, 96)
    shift = rng.integers(-40, 100, 96)
    pre = rng.integers(-(2**40), 2**40, 96)
    post = rng.integers(-(2**20), 2**20, 96)
    args = (acc, 8, 96, 1001, mult, shift, 5, -(2**15), 2**15 - 1)
    np.testing.assert_array_equal(gpu_lib.requantize(*args, pre_bias=pre, post_bias=post),
                                  oracle.requantize(*args, pre_bias=pre, post_bias=post))


@pytest.mark.parametrize("outer,C,inner", [(20000, 12, 1), (3001, 96, 1), (64, 20, 1),
                                           (7, 16, 4096), (3, 24, 3136), (5, 8, 132),
                                           (2, 40, 12)])
def test_requantize_vector_layouts_vs_oracle(gpu_lib, oracle, outer, C, inner):
    """The 16-byte forms: rows of C % 4 == 0 channels (parameters held per
    thread across the grid-stride loop), NCHW planes of inner % 4 == 0 (a
    block per plane; planes whose quads do not fill the last pass) and short
    planes, with channels on the high-word form and on the exact 128-bit
    one."""
    rng = np.random.default_rng(outer + C + inner)
    acc = rng.integers(-(2**31), 2**31, (outer, C, inner)).astype(np.int32)
    mult = rng.integers(0, 2**31, C)
    shift = rng.integers(15, 22, C)  # most outputs inside the int16 range
    mult[::3] = rng.integers(-(2**31) + 1, 0, len(mult[::3]))  # negative: exact form
    shift[1::5] = rng.integers(-3, 0, len(shift[1::5]))  # 31 + shift < 32: exact form
    pre = rng.integers(-(2**28), 2**28, C)
    post = rng.integers(-(2**10), 2**10, C)
    args = (acc, outer, C, inner, mult, shift, -3, -(2**15), 2**15 - 1)
    np.testing.assert_array_equal(gpu_lib.requantize(*args, pre_bias=pre, post_bias=post),
                                  oracle.requantize(*args, pre_bias=pre, post_bias=post))


def test_empty_inputs(gpu_lib):
    z = np.zeros((0,), np.int32)
    assert gpu_lib.rescale(z, 0, 1 << 30, 0, 0, -128, 127).shape == (0,)
    assert gpu_lib.gemm_int(np.zeros((0, 4), np.int32), np.zeros((4, 3), np.int32)).shape == (0, 3)
    out = gpu_lib.gemm_int(np.zeros((2, 0), np.int32), np.zeros((0, 3), np.int32), True)
    np.testing.assert_array_equal(out, np.zeros((2, 3), np.int64))


def test_cfg0_digest(gpu_lib):
    """cfg0 through the drop-in ABI reproduces the reference's output."""
    from quantanything_b200 import configs
    from tests.test_oracle_golden import _digest

    ref = json.loads((GOLDEN / "configs.json").read_text())["cfg0"]
    c = configs.linear_cfg0()
    acc = gpu_lib.gemm_int(c.a - c.a_zp, np.ascontiguousarray(c.w.T), False)
    assert _digest(acc) == ref["acc"]
    out = gpu_lib.requantize(acc, acc.shape[0], acc.shape[1], 1, c.mult, c.shift, c.out_zp,
                             c.qmin, c.qmax, pre_bias=c.bias)
    assert _digest(out) == ref["out"]


def test_cfg1_digest(gpu_lib):
    """cfg1 conv + requantize + SiLU table through the drop-in ABI."""
    from quantanything_b200 import configs
    from tests.test_oracle_golden import _digest

    ref = json.loads((GOLDEN / "configs.json").read_text())["cfg1"]
    c = configs.conv_cfg1()
    acc = gpu_lib.conv2d_int(c.x - c.x_zp, c.w, (1, 1), (1, 1, 1, 1), (1, 1), 1, wide=False)
    assert _digest(acc) == ref["acc"]
    n, co, oh, ow = acc.shape
    mid = gpu_lib.requantize(acc, n, co, oh * ow, c.mult, c.shift, c.mid_zp, c.qmin, c.qmax,
                             pre_bias=c.bias)
    assert _digest(mid) == ref["mid"]
    out = gpu_lib.lut(mid, np.array(ref["table"], np.int32), c.qmin)
    assert _digest(out) == ref["out"]


def test_error_is_reported_not_silent(gpu_lib):
    """A bad geometry raises through the status channel (no silent garbage)."""
    from quantanything_b200.native import KernelLibraryError

    x = np.zeros((1, 4, 5, 5), np.int32)
    w = np.zeros((2, 3, 3, 3), np.int32)  # 4 channels vs 3 per group
    with pytest.raises((KernelLibraryError, ValueError)):
        gpu_lib.conv2d_int(x, w, (1, 1), (1, 1, 1, 1), (1, 1), 1)
