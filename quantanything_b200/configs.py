"""Seeded synthetic workloads of the benchmark configurations.

The reference publishes no dataset-backed throughput numbers for this path,
so every configuration is a seeded synthetic tensor set with the shapes,
ranges and distributions the configuration text names.  The same generators
feed the golden-fixture script, the parity tests and ``bench.py``, so all
three see bit-identical inputs (numpy's ``default_rng`` is platform
independent).

* cfg0 -- one integer Linear: int8 activations [256, 768] with zero point 3,
  int8 per-channel weights [3072, 768], int32 bias, per-channel M0 / shift,
  int8 output with zero point -5.
* cfg1 -- one int8 3x3 conv [32, 64, 56, 56] * [128, 64, 3, 3] with input
  zero point 7, per-channel requantize, then a SiLU lookup table built from
  the conv-output grid (scale 0.1, zero point 0) to the output grid
  (scale 0.05, zero point -20).
"""

from dataclasses import dataclass

import numpy as np


@dataclass
class LinearCase:
    """cfg0 operands (raw integers, before zero-point centring)."""

    a: np.ndarray  # [M, K] int8 values (held as int32), zero point a_zp
    a_zp: int
    w: np.ndarray  # [N, K] int8 symmetric weights (held as int32)
    bias: np.ndarray  # [N] int64
    mult: np.ndarray  # [N] int64 in [2^30, 2^31)
    shift: np.ndarray  # [N] int64 in [8, 12]
    out_zp: int
    qmin: int
    qmax: int


def linear_cfg0(m=256, k=768, n=3072, seed=0):
    """Operands of configuration 0 (seed 0, the reference's CPU case)."""
    rng = np.random.default_rng(seed)
    a = rng.integers(-128, 128, (m, k)).astype(np.int32)
    w = rng.integers(-127, 128, (n, k)).astype(np.int32)
    bias = rng.integers(-(2**20), 2**20, n).astype(np.int64)
    mult = rng.integers(2**30, 2**31, n).astype(np.int64)
    shift = rng.integers(8, 13, n).astype(np.int64)
    return LinearCase(a, 3, w, bias, mult, shift, -5, -128, 127)


@dataclass
class ConvCase:
    """cfg1 operands (raw integers) and the SiLU grid definition."""

    x: np.ndarray  # [N, C, H, W] int8 values (int32), zero point x_zp
    x_zp: int
    w: np.ndarray  # [Cout, C, 3, 3] int8 symmetric (int32)
    bias: np.ndarray  # [Cout] int64
    mult: np.ndarray
    shift: np.ndarray
    mid_scale: float  # grid of the requantized conv output (LUT input)
    mid_zp: int
    out_scale: float  # grid of the SiLU output
    out_zp: int
    qmin: int
    qmax: int
    stride: int = 1
    pad: int = 1


def conv_cfg1(n=32, c=64, h=56, w=56, cout=128, seed=0):
    """Operands of configuration 1 (3x3, stride 1, pad 1, fused SiLU)."""
    rng = np.random.default_rng(seed)
    x = rng.integers(-128, 128, (n, c, h, w)).astype(np.int32)
    wt = rng.integers(-127, 128, (cout, c, 3, 3)).astype(np.int32)
    bias = rng.integers(-(2**18), 2**18, cout).astype(np.int64)
    mult = rng.integers(2**30, 2**31, cout).astype(np.int64)
    shift = rng.integers(8, 13, cout).astype(np.int64)
    return ConvCase(x, 7, wt, bias, mult, shift, 0.1, 0, 0.05, -20, -128, 127)
