"""Host-side quantization maths (parameter derivation).

Same names and meaning as the reference's ``quantization/utils.py``; these
functions run once per layer at preparation time, not on the hot path.
Float -> int conversion of a per-tensor int32 tensor goes through the kernel
library (``native.quantize_f32``), like the reference's fast path
(utils.py:105-109); per-channel weight quantization is host NumPy there too.
"""

from dataclasses import dataclass

import numpy as np

from quantanything_b200 import native

_INT32_MIN, _INT32_MAX = -(2**31), 2**31 - 1


@dataclass
class QParams:
    """Affine parameters of one tensor: ``real = (q - zp) * scale``,
    ``qmin <= q <= qmax`` (utils.py:12-38)."""

    scale: float
    zp: int
    qmin: int
    qmax: int

    def to_dict(self):
        return {"scale": float(self.scale), "zp": int(self.zp),
                "qmin": int(self.qmin), "qmax": int(self.qmax)}

    @classmethod
    def from_dict(cls, d):
        return cls(float(d["scale"]), int(d["zp"]), int(d["qmin"]), int(d["qmax"]))


def parse_quant_type(quant_type):
    """``'int8'`` -> ``(8, True)``, ``'uint16'`` -> ``(16, False)`` (utils.py:41-55)."""
    if quant_type.startswith("uint"):
        return int(quant_type[4:]), False
    if quant_type.startswith("int"):
        return int(quant_type[3:]), True
    raise ValueError(f"Unknown quant_type: {quant_type}")


def quant_range(quant_type):
    """``(qmin, qmax)`` of a type string (utils.py:58-63)."""
    bits, signed = parse_quant_type(quant_type)
    if signed:
        return -(1 << (bits - 1)), (1 << (bits - 1)) - 1
    return 0, (1 << bits) - 1


def calculate_scale_zp(min_val, max_val, quant_type="int8"):
    """Scale and zero point of a calibrated range (utils.py:66-90).

    Signed types are symmetric (zp = 0, scale = max|v| / qmax); unsigned
    types are asymmetric over the range widened to contain 0.  Degenerate
    ranges give scale 1.
    """
    qmin, qmax = quant_range(quant_type)
    _, signed = parse_quant_type(quant_type)
    lo, hi = float(min_val), float(max_val)
    if signed:
        peak = max(abs(lo), abs(hi))
        return (1.0 if peak == 0 else peak / qmax), 0, qmin, qmax
    lo, hi = min(lo, 0.0), max(hi, 0.0)
    if lo == hi:
        return 1.0, 0, qmin, qmax
    scale = (hi - lo) / qmax
    zp = int(np.clip(np.round(-lo / scale), qmin, qmax))
    return scale, zp, qmin, qmax


def _int_dtype(qmin, qmax):
    return np.int32 if _INT32_MIN <= qmin and qmax <= _INT32_MAX else np.int64


def quantize(x, scale, zp, qmin, qmax):
    """Float -> integer, half to even, clipped (utils.py:97-114).

    Scalar scale / zero point on float input with an int32 range runs on the
    GPU kernel library; per-channel parameters run in NumPy on the host.
    """
    x = np.asarray(x)
    dtype = _int_dtype(qmin, qmax)
    if np.ndim(scale) == 0 and np.ndim(zp) == 0:
        if scale == 0:
            return np.full(x.shape, zp, dtype=dtype)
        if dtype == np.int32 and x.dtype in (np.float32, np.float64):
            return native.quantize_f32(x, scale, zp, qmin, qmax)
    scale = np.asarray(scale, dtype=np.float64)
    safe = np.where(scale == 0, 1.0, scale)
    q = np.round(x.astype(np.float64) / safe) + zp
    q = np.where(scale == 0, zp, q)
    return np.clip(q, qmin, qmax).astype(dtype)


def dequantize(q, scale, zp):
    """Integer -> float32, ``(q - zp) * scale`` (utils.py:117-124)."""
    q = np.asarray(q)
    if np.ndim(scale) == 0 and np.ndim(zp) == 0 and q.dtype == np.int32:
        return native.dequantize_f32(q, scale, zp)
    return ((q.astype(np.int64) - zp) * np.asarray(scale, dtype=np.float64)).astype(np.float32)


def fake_quantize(x, scale, zp, qmin, qmax):
    """Quantize then dequantize (utils.py:127-129)."""
    return dequantize(quantize(x, scale, zp, qmin, qmax), scale, zp)


def quantize_multiplier(real_multiplier):
    """``real`` -> ``(M0, shift)`` with ``real = M0 * 2^-(31+shift)`` and
    ``|M0|`` in ``[2^30, 2^31)`` carrying the sign; 0 -> (0, 0)
    (utils.py:132-149).  ``frexp`` gives ``real = f * 2^e`` with f in
    [0.5, 1); M0 = round(f * 2^31), renormalized if it rounds up to 2^31."""
    if real_multiplier < 0:
        m, s = quantize_multiplier(-real_multiplier)
        return -m, s
    if real_multiplier == 0:
        return 0, 0
    frac, exp = np.frexp(real_multiplier)
    m0 = int(np.round(frac * (1 << 31)))
    if m0 >= (1 << 31):
        m0 //= 2
        exp += 1
    return m0, int(-exp)


def quantize_multipliers(real_multipliers):
    """Vectorised :func:`quantize_multiplier` -> two int64 arrays (utils.py:152-159)."""
    flat = np.asarray(real_multipliers, dtype=np.float64).reshape(-1)
    pairs = [quantize_multiplier(float(v)) for v in flat]
    shape = np.shape(real_multipliers)
    mult = np.array([p[0] for p in pairs], dtype=np.int64).reshape(shape)
    shift = np.array([p[1] for p in pairs], dtype=np.int64).reshape(shape)
    return mult, shift


def multiply_by_quantized_multiplier(accum, q_multiplier, shift):
    """``round(accum * M0 * 2^-(31+shift))``, half up, exact for any int64
    input (utils.py:162-167 / qa_kernels.cpp:194-205).  Host utility:
    arbitrary-precision Python integers, element by element."""
    acc = np.asarray(accum, dtype=np.int64)
    mult = np.broadcast_to(np.asarray(q_multiplier, dtype=np.int64), acc.shape)
    sh = np.broadcast_to(np.asarray(shift, dtype=np.int64), acc.shape)
    out = np.empty(acc.shape, dtype=object)
    flat = out.reshape(-1)
    for i, (a, m, s) in enumerate(zip(acc.reshape(-1), mult.reshape(-1), sh.reshape(-1))):
        p = int(a) * int(m)
        t = 31 + int(s)
        flat[i] = (p + (1 << (t - 1))) >> t if t > 0 else p << min(-t, 60)
    return np.clip(out, -(1 << 62), 1 << 62).astype(np.int64)
