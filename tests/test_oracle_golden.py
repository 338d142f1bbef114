"""Pins the C oracle against the reference's own outputs (CPU only).

The fixtures come from the reference's C++ kernels driven by its Python
package (tests/golden/make_golden.py).  An oracle that passes here is a
faithful restatement of the reference on every case the reference tests, so
the GPU tests may use it as the checker on fresh inputs.
"""
import hashlib
import json

import numpy as np
import pytest

from tests import kernel_cases
from tests.conftest import GOLDEN

_CASES = kernel_cases.cases(dict(np.load(GOLDEN / "kernels.npz")))


@pytest.mark.parametrize("name", sorted(_CASES))
def test_oracle_matches_reference(oracle, name):
    got, expected, tol = _CASES[name](oracle)
    kernel_cases.check(got, expected, tol)


def _digest(a):
    a = np.ascontiguousarray(a)
    h = hashlib.sha256()
    h.update(str(a.dtype).encode())
    h.update(str(a.shape).encode())
    h.update(a.tobytes())
    return h.hexdigest()


def test_oracle_cfg0_digest(oracle):
    """cfg0 (256x768x3072 Linear) end to end, against the reference digest."""
    from quantanything_b200 import configs

    ref = json.loads((GOLDEN / "configs.json").read_text())["cfg0"]
    c = configs.linear_cfg0()
    acc = oracle.gemm_int(c.a - c.a_zp, np.ascontiguousarray(c.w.T), False)
    assert _digest(acc) == ref["acc"]
    out = oracle.requantize(acc, acc.shape[0], acc.shape[1], 1, c.mult, c.shift,
                            c.out_zp, c.qmin, c.qmax, pre_bias=c.bias)
    assert _digest(out) == ref["out"]
