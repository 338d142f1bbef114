"""ctypes binding of the kernel library's C ABI (``include/qa_kernels.h``).

Mirrors the reference's kernel boundary (quantization/native.py in the
reference project): the same wrapper names and argument meanings --
``gemm_int``, ``conv2d_int``, ``requantize``, ``rescale``, ``add``, ``mul``,
``lut``, ``quantize_f32``, ``dequantize_f32``, ``gemm_f32``, ``conv2d_f32``
-- over the same 17 C symbols.  Two differences are deliberate:

* there is no NumPy fallback.  The product library is the CUDA build
  ``quantanything_b200/lib/libqa_kernels.so`` (or ``$QA_LIB``); if it cannot
  be loaded every wrapper raises :class:`KernelLibraryError` instead of
  silently computing on the CPU (the reference falls back,
  native.py:141-142);
* every call checks the library's status word (``qa_last_status``) and
  raises :class:`KernelLibraryError` on failure.

:class:`KernelLibrary` wraps any shared object exporting the ABI, so the same
host code can also drive the reference's own CPU build for comparisons.
"""

import ctypes
import os
from pathlib import Path

import numpy as np

_PKG = Path(__file__).resolve().parent
DEFAULT_LIB = _PKG / "lib" / "libqa_kernels.so"

# The 17 symbols and signatures of the reference ABI (native.py:104-128).
_P, _I64, _F64, _INT = ctypes.c_void_p, ctypes.c_int64, ctypes.c_double, ctypes.c_int
REFERENCE_SIGNATURES = {
    "qa_num_threads": (_INT, []),
    "qa_set_num_threads": (None, [_INT]),
    "qa_has_openmp": (_INT, []),
    "qa_gemm_f32": (None, [_I64] * 3 + [_P] * 3),
    "qa_gemm_i16_i32": (None, [_I64] * 3 + [_P] * 3),
    "qa_gemm_i32_i64": (None, [_I64] * 3 + [_P] * 3),
    "qa_conv_f32": (None, [_P] * 3 + [_I64] * 16),
    "qa_conv_i32_i16_i32": (None, [_P] * 3 + [_I64] * 16),
    "qa_conv_i32_i32_i64": (None, [_P] * 3 + [_I64] * 16),
    "qa_requantize_i32": (None, [_P, _P] + [_I64] * 3 + [_P] * 4 + [_I64] * 3),
    "qa_requantize_i64": (None, [_P, _P] + [_I64] * 3 + [_P] * 4 + [_I64] * 3),
    "qa_rescale": (None, [_P, _P] + [_I64] * 7),
    "qa_add": (None, [_P] * 3 + [_I64] * 11),
    "qa_mul": (None, [_P] * 3 + [_I64] * 8),
    "qa_lut": (None, [_P, _P, _I64, _I64, _P, _I64]),
    "qa_quantize_f32": (None, [_P, _P, _I64, _F64, _I64, _I64, _I64]),
    "qa_dequantize_f32": (None, [_P, _P, _I64, _F64, _I64]),
}

# Status / device extensions (no counterpart in the reference).
EXTENSION_SIGNATURES = {
    "qa_last_status": (_INT, []),
    "qa_last_error": (ctypes.c_char_p, []),
    "qa_clear_error": (None, []),
    "qa_set_error_mode": (None, [_INT]),
    "qa_device_count": (_INT, []),
    "qa_set_device": (_INT, [_INT]),
    "qa_get_device": (_INT, []),
}


class KernelLibraryError(RuntimeError):
    """The kernel library is missing, or one of its calls failed."""


def _ptr(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _as_i64(v):
    return np.asarray(v, dtype=np.int64)


def conv_output_size(size, k, stride, pad_begin, pad_end, dilation):
    """Spatial output size of a convolution along one axis (native.py:239)."""
    return (size + pad_begin + pad_end - dilation * (k - 1) - 1) // stride + 1


def conv_geometry(x_shape, w_shape, strides, pads, dilations, groups):
    """Resolves the 16 integers of the conv ABI (native.py:244-257).

    Returns ``(n, c, h, w, cout, kh, kw, sh, sw, pt, pl, dh, dw, oh, ow)``
    and raises ``ValueError`` on inconsistent channel / group counts, the
    reference's only shape check.
    """
    n, c, h, wd = x_shape
    cout, cg, kh, kw = w_shape
    if c != cg * groups or cout % groups:
        raise ValueError(
            f"conv shape mismatch: input C={c}, weight={tuple(w_shape)}, "
            f"groups={groups}"
        )
    sh, sw = strides
    dh, dw = dilations
    pt, pl, pb, pr = pads
    oh = conv_output_size(h, kh, sh, pt, pb, dh)
    ow = conv_output_size(wd, kw, sw, pl, pr, dw)
    return n, c, h, wd, cout, kh, kw, sh, sw, pt, pl, dh, dw, oh, ow


def accumulator_is_wide(num_bits, reduction_size):
    """Whether a dot product needs the int64 accumulator (native.py:363-373).

    The int32 path holds operands as int16, so it is valid only when the
    zero-point-centred operands fit int16 (``num_bits <= 15``) and
    ``2^(2·bits) · K`` stays below 2^31.
    """
    if num_bits > 15:
        return True
    return ((1 << num_bits) ** 2) * int(reduction_size) >= (1 << 31)


class KernelLibrary:
    """A loaded shared object exporting the 17-symbol kernel ABI."""

    def __init__(self, path):
        self.path = str(path)
        try:
            lib = ctypes.CDLL(self.path)
        except OSError as exc:
            raise KernelLibraryError(f"cannot load {self.path}: {exc}") from exc
        for name, (res, args) in REFERENCE_SIGNATURES.items():
            try:
                fn = getattr(lib, name)
            except AttributeError as exc:
                raise KernelLibraryError(f"{self.path} lacks {name}") from exc
            fn.restype, fn.argtypes = res, args
        self.has_status = all(hasattr(lib, n) for n in EXTENSION_SIGNATURES)
        if self.has_status:
            for name, (res, args) in EXTENSION_SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype, fn.argtypes = res, args
            lib.qa_set_error_mode(0)  # record, so failures become exceptions
        self._lib = lib

    # ------------------------------------------------------------ plumbing --
    @property
    def raw(self):
        """The underlying :class:`ctypes.CDLL`."""
        return self._lib

    def check(self, what):
        """Raises if the library recorded a failure for the last call."""
        if self.has_status and self._lib.qa_last_status() != 0:
            msg = self._lib.qa_last_error().decode(errors="replace")
            self._lib.qa_clear_error()
            raise KernelLibraryError(f"{what}: {msg}")

    def set_device(self, ordinal):
        """Binds the calling host thread's library work to GPU ``ordinal``
        (host-pointer calls, and the device entry points' launches)."""
        if self.has_status:
            rc = self._lib.qa_set_device(int(ordinal))
            if rc != 0:
                self.check("qa_set_device")

    def num_threads(self):
        return self._lib.qa_num_threads()

    def has_openmp(self):
        return self._lib.qa_has_openmp()

    def set_num_threads(self, n):
        self._lib.qa_set_num_threads(int(n))

    # ---------------------------------------------------------------- GEMM --
    def gemm_f32(self, a, b):
        """``a[M,K] @ b[K,N]`` in float32 (native.py:207)."""
        a, b = _c(a, np.float32), _c(b, np.float32)
        if a.shape[1] != b.shape[0]:
            raise ValueError(f"gemm_f32: inner dimensions differ ({a.shape} @ {b.shape})")
        out = np.empty((a.shape[0], b.shape[1]), dtype=np.float32)
        self._lib.qa_gemm_f32(a.shape[0], b.shape[1], a.shape[1], _ptr(a),
                              _ptr(b), _ptr(out))
        self.check("qa_gemm_f32")
        return out

    def gemm_int(self, a, b, wide=False):
        """Integer ``a[M,K] @ b[K,N]``: int32 accumulator, int64 if ``wide``
        (native.py:219)."""
        m, k = a.shape
        n = b.shape[1]
        if b.shape[0] != k:
            raise ValueError(f"gemm_int: inner dimensions differ ({a.shape} @ {b.shape})")
        if wide:
            a, b = _c(a, np.int32), _c(b, np.int32)
            out = np.empty((m, n), dtype=np.int64)
            self._lib.qa_gemm_i32_i64(m, n, k, _ptr(a), _ptr(b), _ptr(out))
            self.check("qa_gemm_i32_i64")
        else:
            a, b = _c(a, np.int16), _c(b, np.int16)
            out = np.empty((m, n), dtype=np.int32)
            self._lib.qa_gemm_i16_i32(m, n, k, _ptr(a), _ptr(b), _ptr(out))
            self.check("qa_gemm_i16_i32")
        return out

    # ---------------------------------------------------------------- conv --
    def conv2d_f32(self, x, w, strides=(1, 1), pads=(0, 0, 0, 0),
                   dilations=(1, 1), groups=1):
        """Float32 NCHW convolution, OIHW weights (native.py:280)."""
        x, w = _c(x, np.float32), _c(w, np.float32)
        g = conv_geometry(x.shape, w.shape, strides, pads, dilations, groups)
        n, c, h, wd, cout, kh, kw, sh, sw, pt, pl, dh, dw, oh, ow = g
        out = np.empty((n, cout, oh, ow), dtype=np.float32)
        self._lib.qa_conv_f32(_ptr(x), _ptr(w), _ptr(out), n, c, h, wd, cout,
                              kh, kw, sh, sw, pt, pl, dh, dw, groups, oh, ow)
        self.check("qa_conv_f32")
        return out

    def conv2d_int(self, x, w, strides=(1, 1), pads=(0, 0, 0, 0),
                   dilations=(1, 1), groups=1, wide=False):
        """Integer NCHW convolution of zero-point-centred operands
        (native.py:315); int32 accumulators, int64 when ``wide``."""
        x = _c(x, np.int32)
        g = conv_geometry(x.shape, w.shape, strides, pads, dilations, groups)
        n, c, h, wd, cout, kh, kw, sh, sw, pt, pl, dh, dw, oh, ow = g
        args = (n, c, h, wd, cout, kh, kw, sh, sw, pt, pl, dh, dw, groups, oh, ow)
        if wide:
            w = _c(w, np.int32)
            out = np.empty((n, cout, oh, ow), dtype=np.int64)
            self._lib.qa_conv_i32_i32_i64(_ptr(x), _ptr(w), _ptr(out), *args)
            self.check("qa_conv_i32_i32_i64")
        else:
            w = _c(w, np.int16)
            out = np.empty((n, cout, oh, ow), dtype=np.int32)
            self._lib.qa_conv_i32_i16_i32(_ptr(x), _ptr(w), _ptr(out), *args)
            self.check("qa_conv_i32_i16_i32")
        return out

    # ---------------------------------------------------------- requantize --
    def requantize(self, acc, outer, channels, inner, mult, shift, zp, qmin,
                   qmax, pre_bias=None, post_bias=None):
        """Per-channel fixed-point requantization of ``acc`` viewed as
        ``[outer, channels, inner]`` (native.py:377)."""
        mult = _c(np.broadcast_to(_as_i64(mult), (channels,)), np.int64)
        shift = _c(np.broadcast_to(_as_i64(shift), (channels,)), np.int64)
        wide = acc.dtype == np.int64
        acc = _c(acc, np.int64 if wide else np.int32)
        out = np.empty(acc.shape, dtype=np.int32)
        pre = (None if pre_bias is None else
               _c(np.broadcast_to(_as_i64(pre_bias), (channels,)), np.int64))
        post = (None if post_bias is None else
                _c(np.broadcast_to(_as_i64(post_bias), (channels,)), np.int64))
        fn = self._lib.qa_requantize_i64 if wide else self._lib.qa_requantize_i32
        fn(_ptr(acc), _ptr(out), outer, channels, inner, _ptr(mult),
           _ptr(shift), _ptr(pre), _ptr(post), int(zp), int(qmin), int(qmax))
        self.check("qa_requantize")
        return out

    # -------------------------------------------------------- element-wise --
    def rescale(self, x, zp_in, mult, shift, zp_out, qmin, qmax):
        """``clip(mbqm(x - zp_in) + zp_out)`` element-wise (native.py:444)."""
        x = _c(x, np.int32)
        out = np.empty_like(x)
        self._lib.qa_rescale(_ptr(x), _ptr(out), x.size, int(zp_in), int(mult),
                             int(shift), int(zp_out), int(qmin), int(qmax))
        self.check("qa_rescale")
        return out

    def add(self, a, b, za, ma, sa, zb, mb, sb, zp_out, qmin, qmax, sign=1):
        """Rescale both operands to the output grid and add (or subtract)
        (native.py:465)."""
        a, b = np.broadcast_arrays(a, b)
        a, b = _c(a, np.int32), _c(b, np.int32)
        out = np.empty_like(a)
        self._lib.qa_add(_ptr(a), _ptr(b), _ptr(out), a.size, int(za), int(ma),
                         int(sa), int(zb), int(mb), int(sb), int(sign),
                         int(zp_out), int(qmin), int(qmax))
        self.check("qa_add")
        return out

    def mul(self, a, b, za, zb, mult, shift, zp_out, qmin, qmax):
        """``clip(mbqm((a - za)(b - zb)) + zp_out)`` (native.py:496)."""
        a, b = np.broadcast_arrays(a, b)
        a, b = _c(a, np.int32), _c(b, np.int32)
        out = np.empty_like(a)
        self._lib.qa_mul(_ptr(a), _ptr(b), _ptr(out), a.size, int(za), int(zb),
                         int(mult), int(shift), int(zp_out), int(qmin),
                         int(qmax))
        self.check("qa_mul")
        return out

    def lut(self, x, table, offset):
        """``table[clip(x - offset, 0, len(table) - 1)]`` (native.py:521)."""
        table = _c(table, np.int32)
        x = _c(x, np.int32)
        out = np.empty_like(x)
        self._lib.qa_lut(_ptr(x), _ptr(out), x.size, int(offset), _ptr(table),
                         len(table))
        self.check("qa_lut")
        return out

    # ------------------------------------------------- float <-> integer --
    def quantize_f32(self, x, scale, zp, qmin, qmax):
        """Per-tensor float -> int32, half to even (native.py:536)."""
        x = _c(x, np.float32)
        out = np.empty(x.shape, dtype=np.int32)
        self._lib.qa_quantize_f32(_ptr(x), _ptr(out), x.size, float(scale),
                                  int(zp), int(qmin), int(qmax))
        self.check("qa_quantize_f32")
        return out

    def dequantize_f32(self, q, scale, zp):
        """Per-tensor int32 -> float32 (native.py:549)."""
        q = _c(q, np.int32)
        out = np.empty(q.shape, dtype=np.float32)
        self._lib.qa_dequantize_f32(_ptr(q), _ptr(out), q.size, float(scale),
                                    int(zp))
        self.check("qa_dequantize_f32")
        return out


# ------------------------------------------------------- default library --
_default = None
_load_error = None


def library_path():
    """Path of the product library: ``$QA_LIB`` or the in-tree CUDA build."""
    return Path(os.environ.get("QA_LIB") or DEFAULT_LIB)


def get_library():
    """The loaded product library; raises :class:`KernelLibraryError` (never
    falls back) when it is missing or fails to load."""
    global _default, _load_error
    if _default is None:
        path = library_path()
        if not path.exists():
            _load_error = (f"{path} not found; build it with "
                           "`python -c 'import __graft_entry__ as g; g.build()'`")
            raise KernelLibraryError(_load_error)
        try:
            _default = KernelLibrary(path)
        except KernelLibraryError as exc:
            _load_error = str(exc)
            raise
    return _default


def available():
    """True when the product library loads."""
    try:
        get_library()
        return True
    except KernelLibraryError:
        return False


def load_error():
    """Why the product library did not load (None when it did)."""
    return _load_error


def _delegate(name):
    def fn(*args, **kwargs):
        return getattr(get_library(), name)(*args, **kwargs)

    fn.__name__ = name
    fn.__doc__ = getattr(KernelLibrary, name).__doc__
    return fn


gemm_f32 = _delegate("gemm_f32")
gemm_int = _delegate("gemm_int")
conv2d_f32 = _delegate("conv2d_f32")
conv2d_int = _delegate("conv2d_int")
requantize = _delegate("requantize")
rescale = _delegate("rescale")
add = _delegate("add")
mul = _delegate("mul")
lut = _delegate("lut")
quantize_f32 = _delegate("quantize_f32")
dequantize_f32 = _delegate("dequantize_f32")


def set_num_threads(n):
    """Accepted for interface parity; GPU work is not host-threaded."""
    get_library().set_num_threads(n)
