"""The 16-bit epilogue's shortcut forms of the reference's mbqm
(qa_kernels.cpp:194-205), restated in Python integers exactly as
csrc/qa_fixedpoint.cuh computes them (64-bit two's-complement words), must
equal the exact 128-bit definition on their stated domains."""
import numpy as np

M64 = (1 << 64) - 1


def _s64(v):
    v &= M64
    return v - (1 << 64) if v >> 63 else v


def mbqm_exact(x, m, s):
    ts = 31 + s
    p = x * m
    if ts > 0:
        ts = min(ts, 120)
        return (p + (1 << (ts - 1))) >> ts
    return p << min(-ts, 60)


def requant_hi32(x, m, ts):
    """requant_hi32 of qa_fixedpoint.cuh without the bias / clamp."""
    xh = _s64(x) >> 32
    xlm = (x & 0xFFFFFFFF) * m  # < 2^63: unsigned 64-bit product
    assert xlm < 1 << 64
    if ts == 32:
        return _s64(xh * m + ((xlm + (1 << 31)) >> 32))
    c = _s64(xh * m + (xlm >> 32) + (1 << (ts - 33)))
    assert -(1 << 63) <= xh * m + (xlm >> 32) + (1 << (ts - 33)) < 1 << 63
    return c >> (ts - 32)


def mbqm_small(x, m, ts):
    v = x * m + (1 << (ts - 1))
    assert -(1 << 63) <= v < 1 << 63
    return v >> ts


def test_hi32_form_equals_mbqm():
    rng = np.random.default_rng(0)
    xs = [0, 1, -1, (1 << 63) - 1, -(1 << 63), (1 << 32) - 1, -(1 << 32), 1 << 40, -(1 << 40) - 7]
    xs += [int(v) for v in rng.integers(-(1 << 63), (1 << 63) - 1, 400, dtype=np.int64)]
    xs += [int(v) for v in rng.integers(-(1 << 45), 1 << 45, 400)]
    ms = [0, 1, (1 << 30), (1 << 31) - 1] + [int(v) for v in rng.integers(1 << 30, 1 << 31, 20)]
    for ts in [32, 33, 34, 40, 47, 63, 64, 65, 80, 94]:
        for m in ms:
            for x in xs:
                assert requant_hi32(x, m, ts) == mbqm_exact(x, m, ts - 31), (x, m, ts)


def test_small_form_equals_mbqm():
    rng = np.random.default_rng(1)
    xs = [0, 1, -1, 65535, -65535, (1 << 31) - 1, -(1 << 31) + 1]
    xs += [int(v) for v in rng.integers(-65536, 65536, 300)]
    ms = [0, 1, -1, (1 << 31) - 1, -(1 << 31) + 1] + [int(v) for v in
                                                      rng.integers(-(1 << 31) + 1, 1 << 31, 20)]
    for s in [-30, -29, -1, 0, 5, 12, 20, 31]:
        for m in ms:
            for x in xs:
                assert mbqm_small(x, m, 31 + s) == mbqm_exact(x, m, s), (x, m, s)
