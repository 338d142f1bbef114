"""NumPy stand-ins for the device float-pass entry points (qa_f32_*), for
CPU tests of the device calibration's host logic.

The calibrator hands these the data pointers of CPU tensors, so each stand
in reads and writes host memory through the same pointers, sizes, strides
and range slots the CUDA kernels get.  Convolutions run the C oracle's
qa_conv_f32.  Test infrastructure only.
"""
import ctypes

import numpy as np

from quantanything_b200 import float_ops


def _arr(ptr, n, dtype=np.float32):
    if n <= 0:
        return np.empty(0, dtype)
    ct = np.ctypeslib.as_ctypes_type(dtype)
    return np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ct)), shape=(int(n),))


def _keys(v):
    u = np.ascontiguousarray(v, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000).astype(np.uint64)


def _offsets(shape, strides):
    off = np.zeros((), np.int64)
    for d, (n, s) in enumerate(zip(shape, strides)):
        idx = np.arange(n, dtype=np.int64) * s
        off = off[..., None] + idx if d else idx
    return np.asarray(off).reshape(-1)


def _strided(ptr, shape, strides):
    off = _offsets(shape, strides)
    if off.size == 0:
        return np.empty(0, np.float32), off
    lo = int(off.min())
    base = _arr(ptr + 4 * lo, int(off.max()) - lo + 1)
    return base, off - lo


class FakeFloatKernels:
    _qa_calib_declared = True  # plain Python callables: no ctypes prototypes to declare

    def __init__(self, oracle_raw):
        self.oracle = oracle_raw
        self.calls = []

    # -- plumbing the calibrator expects of a loaded library
    def qa_last_error(self):
        return b""

    def qa_clear_error(self):
        pass

    def _fold(self, rng, values):
        if rng is None or np.size(values) == 0:
            return
        k = _keys(np.asarray(values).reshape(-1))
        slot = _arr(rng, 2, np.uint32)
        slot[0] = min(int(slot[0]), int(k.min()))
        slot[1] = max(int(slot[1]), int(k.max()))

    @staticmethod
    def _dims(rank, shape, *strides):
        r = int(rank)
        return [int(shape[i]) for i in range(r)], [[int(s[i]) for i in range(r)] for s in strides]

    # -- the entry points
    def qa_f32_map_dev(self, x, y, n, op, p0, p1, rng, st):
        self.calls.append("map")
        v = _arr(x, n).astype(np.float64)
        f32 = _arr(x, n)
        out = {
            0: lambda: f32,
            1: lambda: 1.0 / (1.0 + np.exp(-v)),
            2: lambda: np.maximum(f32, 0),
            3: lambda: np.where(f32 >= 0, f32, np.float32(p0) * f32),
            4: lambda: np.tanh(f32),
            5: lambda: np.clip(np.float32(p0) * f32 + np.float32(p1), 0, 1),
            6: lambda: f32 * np.clip(f32 / np.float32(6) + np.float32(0.5), 0, 1),
            7: lambda: np.where(v > 0, v, p0 * np.expm1(np.minimum(v, 0))),
            8: lambda: np.logaddexp(0, v),
            9: lambda: np.abs(f32),
            10: lambda: -f32,
            11: lambda: np.sqrt(f32),
            12: lambda: np.exp(v),
            13: lambda: float_ops.erf_as(v),
            14: lambda: 0.5 * v * (1 + float_ops.erf_as(v / np.sqrt(2))),
            15: lambda: 0.5 * v * (1 + np.tanh(np.sqrt(2 / np.pi) * (v + 0.044715 * v**3))),
            16: lambda: np.clip(f32, np.float32(p0), np.float32(p1)),
        }[int(op)]().astype(np.float32)
        _arr(y, n)[:] = out
        self._fold(rng, out)
        return 0

    def qa_f32_binary_dev(self, a, b, y, rank, shape, sa, sb, op, rng, st):
        self.calls.append("binary")
        dims, (sa, sb) = self._dims(rank, shape, sa, sb)
        ab, ao = _strided(a, dims, sa)
        bb, bo = _strided(b, dims, sb)
        av, bv = ab[ao], bb[bo]
        fn = [np.add, np.subtract, np.multiply, np.divide, np.maximum, np.minimum][int(op)] \
            if int(op) < 6 else None
        out = fn(av, bv) if fn else np.power(av.astype(np.float64), bv.astype(np.float64))
        out = out.astype(np.float32)
        _arr(y, out.size)[:] = out
        self._fold(rng, out)
        return 0

    def qa_f32_copy_dev(self, x, y, rank, shape, sx, sy, rng, st):
        self.calls.append("copy")
        dims, (sx, sy) = self._dims(rank, shape, sx, sy)
        xb, xo = _strided(x, dims, sx)
        yb, yo = _strided(y, dims, sy)
        v = xb[xo].copy()
        yb[yo] = v
        self._fold(rng, v)
        return 0

    def qa_f32_fill_dev(self, y, n, value, rng, st):
        self.calls.append("fill")
        _arr(y, n)[:] = np.float32(value)
        self._fold(rng, np.float32([value]))
        return 0

    def qa_f32_range_dev(self, x, n, rng, st):
        self.calls.append("range")
        self._fold(rng, _arr(x, n))
        return 0

    def qa_f32_range_decode_dev(self, rng, out, count, st):
        k = _arr(rng, 2 * count, np.uint32).astype(np.uint64)
        u = np.where(k & 0x80000000, k & 0x7FFFFFFF, (~k) & 0xFFFFFFFF).astype(np.uint32)
        f = u.view(np.float32).reshape(-1, 2).copy()
        kk = k.reshape(-1, 2)
        f[kk[:, 0] == 0xFFFFFFFF, 0] = np.inf
        f[kk[:, 1] == 0, 1] = -np.inf
        f[:, 1] = -f[:, 1]
        _arr(out, 2 * count)[:] = f.reshape(-1)
        return 0

    def qa_f32_gemm_dev(self, A, B, C, batch, M, N, K, ab, am, ak, bb, bk, bn, alpha, rng, st):
        self.calls.append("gemm")
        out = np.empty((batch, M, N), np.float32)
        for z in range(batch):
            abase, aoff = _strided(A + 4 * z * ab, (M, K), (am, ak))
            bbase, boff = _strided(B + 4 * z * bb, (K, N), (bk, bn))
            g = np.matmul(abase[aoff].reshape(M, K), bbase[boff].reshape(K, N))
            out[z] = g if np.float32(alpha) == 1 else np.float32(alpha) * g
        _arr(C, out.size)[:] = out.reshape(-1)
        self._fold(rng, out)
        return 0

    def qa_f32_conv_dev(self, x, w, y, *geom_and_stream):
        self.calls.append("conv")
        geom = geom_and_stream[:16]
        self.oracle.qa_conv_f32(ctypes.c_void_p(x), ctypes.c_void_p(w), ctypes.c_void_p(y),
                                *[ctypes.c_int64(int(g)) for g in geom])
        return 0

    def qa_f32_softmax_dev(self, x, y, rows, cols, rng, st):
        self.calls.append("softmax")
        v = _arr(x, rows * cols).reshape(rows, cols).astype(np.float64)
        e = np.exp(v - v.max(axis=1, keepdims=True))
        out = (e / e.sum(axis=1, keepdims=True)).astype(np.float32)
        _arr(y, out.size)[:] = out.reshape(-1)
        self._fold(rng, out)
        return 0

    def qa_f32_layernorm_dev(self, x, gamma, beta, y, rows, D, eps, rng, st):
        self.calls.append("layernorm")
        v = _arr(x, rows * D).reshape(rows, D).astype(np.float64)
        mean = v.mean(axis=1, keepdims=True)
        var = ((v - mean) ** 2).mean(axis=1, keepdims=True)
        t = (v - mean) / np.sqrt(var + eps) * _arr(gamma, D)
        if beta:
            t = t + _arr(beta, D)
        out = t.astype(np.float32)
        _arr(y, out.size)[:] = out.reshape(-1)
        self._fold(rng, out)
        return 0

    def qa_f32_maxpool_dev(self, x, y, NC, H, W, kh, kw, sh, sw, pt, pl, dh, dw, OH, OW, rng,
                           st):
        self.calls.append("maxpool")
        v = _arr(x, NC * H * W).reshape(NC, H, W)
        out = np.full((NC, OH, OW), -np.inf, np.float32)
        for a in range(kh):
            for b in range(kw):
                for oy in range(OH):
                    iy = oy * sh - pt + a * dh
                    if not 0 <= iy < H:
                        continue
                    for ox in range(OW):
                        ix = ox * sw - pl + b * dw
                        if 0 <= ix < W:
                            out[:, oy, ox] = np.maximum(out[:, oy, ox], v[:, iy, ix])
        _arr(y, out.size)[:] = out.reshape(-1)
        self._fold(rng, out)
        return 0

    def qa_f32_plane_mean_dev(self, x, y, NC, HW, rng, st):
        self.calls.append("mean")
        out = _arr(x, NC * HW).reshape(NC, HW).mean(axis=1).astype(np.float32)
        _arr(y, NC)[:] = out
        self._fold(rng, out)
        return 0


class FakeLibrary:
    def __init__(self, oracle):
        self.raw = FakeFloatKernels(oracle.raw)
