"""Device-resident, fused execution of 16-bit (int16) graphs -- and of uint8
graphs, whose asymmetric weights do not fit the 8-bit tensor path.

The reference runs an int16 graph with every Conv and Gemm on its wide
route: int32 operands, int64 accumulators (``native.accumulator_is_wide``,
native.py:363-373 -> qa_conv_i32_i32_i64 / qa_gemm_i32_i64,
qa_kernels.cpp:260-263, 281-284), then requantizes with the 128-bit
``mbqm`` (qa_kernels.cpp:188-228).  ResidentNet16 computes the same
integers with the activations resident in HBM as two NHWC byte planes per
tensor (low byte ``v & 0xFF``, high byte ``v >> 8``):

* dense Conv / Gemm run on the tensor cores as four 8-bit products per
  K-step (lo*lo, lo*hi, hi*lo, hi*hi) into three int32 TMEM accumulators
  that the epilogue combines in int64 -- exact, and so identical to the
  reference's int64 accumulation, while K * 255 * 255 < 2^31 (K < 33025;
  YOLOv8n-cls's largest K is 1280) -- with requantize, the 65536-entry
  activation LUT, the residual Add and the rescaled Concat copy fused into
  the same launch (``qa_conv16_fused_dev``); grouped / depthwise layers run
  the same epilogue on CUDA cores;
* Split / Flatten are views, Concat inputs are written into their slice,
  GlobalAveragePool and the Softmax fallback are one kernel each, and the
  graph input is quantized straight into the planes.

The planner is ResidentNet's (same fusion decisions); only the storage,
the weight packing and the launches differ.
"""

import ctypes

import numpy as np
import torch

from quantanything_b200.resident import (
    FusedConvDesc,
    ResidentNet,
    UnsupportedGraph,
    View,
    _check,
    _round_up,
)

_I64 = ctypes.c_int64
_P = ctypes.c_void_p
_D = ctypes.c_double


class FusedConv16Desc(ctypes.Structure):
    """ctypes mirror of ``qa_fused_conv16_desc`` (include/qa_kernels.h)."""

    _fields_ = [("base", FusedConvDesc), ("x_plane", _I64), ("res_plane", _I64),
                ("out_plane", _I64), ("out2_plane", _I64), ("lut16", _P),
                ("w_planes", _I64)]


_DEV16_SIGNATURES = {
    "qa_conv16_fused_dev": (ctypes.c_int, [ctypes.POINTER(FusedConv16Desc), _P]),
    "qa_quantize_to_planes16_dev": (ctypes.c_int, [_P, _P, _I64, _I64, _I64, _I64, _I64, _I64,
                                                   _D, _I64, _I64, _I64, _P]),
    "qa_gap16_dev": (ctypes.c_int, [_P] + [_I64] * 11 + [_P, _I64, _I64, _P]),
    "qa_softmax16_dev": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, _D, _I64, _D, _I64, _I64,
                                        _I64, _P, _P, _D, _I64, _P]),
    "qa_lut16_dev": (ctypes.c_int, [_P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _I64, _P,
                                    _I64, _P]),
    "qa_add16_dev": (ctypes.c_int, [_P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64]
                     + [_I64] * 12 + [_P]),
    "qa_rescale16_dev": (ctypes.c_int, [_P, _I64, _I64, _P, _I64, _I64] + [_I64] * 9 + [_P]),
    "qa_maxpool16_dev": (ctypes.c_int, [_P, _I64, _I64, _P, _I64, _I64] + [_I64] * 15 + [_P]),
    "qa_mul16_dev": (ctypes.c_int, [_P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64]
                     + [_I64] * 9 + [_P]),
    "qa_bn16_dev": (ctypes.c_int, [_P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _P,
                                   _I64, _I64, _I64, _P]),
}


def device_api16(lib):
    """Declares the 16-bit device-pointer entry points on a KernelLibrary."""
    raw = lib.raw
    if not getattr(raw, "_qa_dev16_declared", False):
        for name, (res, args) in _DEV16_SIGNATURES.items():
            fn = getattr(raw, name)
            fn.restype, fn.argtypes = res, args
        raw._qa_dev16_declared = True
    return raw


UINT16_SHIFT = 32768


def shifted_container(container, shift=UINT16_SHIFT):
    """A view of ``container`` whose activations live ``shift`` lower: every
    activation QParams (zp, qmin, qmax), activation table (values and index
    offset) and quantized constant moves by ``-shift``; weights, scales,
    multipliers and biases are untouched.  The reference's integer steps
    read activations only through ``v - zp`` (contractions, Add, Mul,
    Concat rescale, GAP, the float fallbacks), ``v - qmin`` (tables), order
    (MaxPool) or write ``clamp(. + zp, qmin, qmax)`` (requantize), so every
    value of the shifted graph is the original minus ``shift``: a uint16
    graph ([0, 65535]) runs on signed int16 planes."""
    import copy

    from quantanything_b200.utils import QParams

    def sq(qp):
        return QParams(qp.scale, int(qp.zp) - shift, int(qp.qmin) - shift, int(qp.qmax) - shift)

    c = copy.copy(container)
    c.qparams = {k: sq(v) for k, v in container.qparams.items()}
    c._const_q = {k: np.asarray(v, np.int64) - shift for k, v in container._const_q.items()}
    layers = {}
    for name, layer in container.quant_layers.items():
        sl = copy.copy(layer)
        sl.in_qp = [sq(q) for q in layer.in_qp]
        sl.out_qp = [sq(q) for q in layer.out_qp]
        if getattr(layer, "lut", None) is not None:
            sl.lut = (np.asarray(layer.lut, np.int64) - shift).astype(np.int32)
            sl.lut_offset = int(layer.lut_offset) - shift
        layers[name] = sl
    c.quant_layers = layers
    return c


class ResidentNet16(ResidentNet):
    """Fused device-resident integer inference of a prepared int16 container
    (also uint8, and uint16 through ``shifted_container``)."""

    # the persistent kernel runs column tiles up to 128 (two TMEM accumulator
    # sets of 3 x BN columns up to 64, one set at 128); measured on B200 the
    # YOLOv8n-cls step is the same at 64 and 128 (the 1x1 layers lose the
    # shared-memory table at 128 what the 3x3 ones gain), 7% slower at 32
    _max_block_n = 64

    def __init__(self, container, batch, device=None):
        self._planes = []  # (low plane start, plane bytes) of every allocation
        self._lut16 = {}   # int32 table address -> int16 device copy
        layer0 = container.layers[0]
        # uint16: activations stored 32768 lower (signed int16 planes); the
        # centred weights span 17 bits and take three byte planes
        self._act_shift = UINT16_SHIFT if (layer0.num_bits == 16 and not layer0.signed) else 0
        self._w_planes = 3 if self._act_shift else 2
        self._orig = container
        if self._act_shift:
            container = shifted_container(container, self._act_shift)
        super().__init__(container, batch, device, fuse_input=False)
        device_api16(self.lib)
        self._descs = {}

    # ---------------------------------------------------------- storage --
    def _check_bits(self):
        # uint8 graphs (asymmetric activations and weights) take this route
        # too: their centred weights span [-255, 255], past int8 but within
        # int16, and a uint8 value is an int16 with a zero high byte
        if not (self.bits == 16 or (self.bits == 8 and not self.signed)):
            raise UnsupportedGraph("ResidentNet16 runs int16, uint16 and uint8 graphs")

    def _operand_bits(self):
        return 16

    def _weight_bits(self):
        return 17 if self._w_planes == 3 else 16

    def output_int(self):
        """int32 graph output of the last run on the reference's grid (a
        uint16 graph's shifted activations moved back: a new tensor)."""
        return self.out_q + self._act_shift if self._act_shift else self.out_q

    def output_qparams(self):
        return self._orig.qparams[self.graph.outputs[0]]

    def _new_view(self, N, H, W, C, qp, pix_stride=None):
        stride = pix_stride or (C if C % 16 == 0 else _round_up(C, 16))
        plane = _round_up(N * H * W * stride, 256)
        buf = self._alloc(2 * plane)
        self._planes.append((buf.data_ptr(), plane))
        return View(buf, 0, stride, N, H, W, C, True, qp, plane)

    def _plane_of(self, ptr):
        """Plane distance of the allocation holding device address ``ptr``."""
        for start, plane in self._planes:
            if start <= ptr < start + plane:
                return plane
        raise AssertionError(f"address {ptr:#x} is not in a planned 16-bit tensor")

    def _plan_contraction(self, layer, layers, fused_away, patch=0):
        super()._plan_contraction(layer, layers, fused_away, patch)
        # desc.fast (16-bit meaning): every channel takes the kernel's exact
        # high-word requantize, 0 <= M0 < 2^31 and 32 <= 31 + shift <= 94
        step = self.steps[-1][1]
        cout = int(step.desc.Cout)
        mult = np.broadcast_to(np.asarray(layer.q_mult, np.int64), (cout,))
        ts = 31 + np.broadcast_to(np.asarray(layer.shift, np.int64), (cout,))
        step.desc.fast = int(bool(np.all((mult >= 0) & (mult < 2**31) & (ts >= 32)
                                         & (ts <= 94))))

    def _upload_weights(self, packed):
        # [rows, kp] -> [2][rows][kp] bytes (low plane, high plane) for int16
        # weights, [3][rows][kp] (bytes 0, 1, sign byte) for 17-bit ones
        v = packed.astype(np.int64)
        planes = [(v >> (8 * i)) & 0xFF for i in range(self._w_planes)]
        return self._dev(np.concatenate([p.astype(np.uint8) for p in planes]), np.uint8)

    def _desc16(self, step):
        d16 = self._descs.get(id(step))
        if d16 is None:
            d = step.desc
            d16 = FusedConv16Desc()
            d16.base = d
            d16.x_plane = self._plane_of(d.x)
            d16.res_plane = self._plane_of(d.res) if d.res else 0
            d16.out_plane = self._plane_of(d.out) if d.out else 0
            d16.out2_plane = self._plane_of(d.out2) if d.out2 else 0
            lut = self._lut_as_int16(d.lut, d.lut_len) if d.lut else None
            d16.lut16 = lut.data_ptr() if lut is not None else None
            d16.w_planes = self._w_planes
            self._descs[id(step)] = d16
        return d16

    def _lut_as_int16(self, ptr, n):
        """int16 copy of a planned int32 activation table (the kernel keeps
        it in shared memory), or None when it does not fit int16.  Made on
        the first (eager) launch, never inside a graph capture."""
        if ptr in self._lut16:
            return self._lut16[ptr]
        src = next(t for t in self._keep if t.data_ptr() == ptr)
        t = None
        if n <= 65536 and int(src.min()) >= -32768 and int(src.max()) <= 32767:
            t = src.to(torch.int16)
            self._keep.append(t)
        self._lut16[ptr] = t
        return t

    # ----------------------------------------------------------- launch --
    def _launch_all(self, stream, on_step=None):
        raw = self.lib.raw
        raw.qa_set_device(self.device.index)
        st = ctypes.c_void_p(stream)
        n = 0
        for kind, payload in self.steps:
            if kind == "quantize":
                v, qp = self._in_view, self.c.qparams[payload]
                N, C, H, W = self.in_shape
                rc = raw.qa_quantize_to_planes16_dev(self.x_dev.data_ptr(), v.ptr, v.plane, N, C,
                                                     H, W, v.pix_stride, float(qp.scale), qp.zp,
                                                     qp.qmin, qp.qmax, st)
            elif kind == "conv":
                rc = raw.qa_conv16_fused_dev(ctypes.byref(self._desc16(payload)), st)
            elif kind == "rescale":
                concat, idx, src, dst = payload
                m, s = concat._mult[idx]
                qp, o = concat.in_qp[idx], concat.out_qp[0]
                rc = raw.qa_rescale16_dev(src.ptr, src.plane, src.pix_stride, dst.ptr, dst.plane,
                                          dst.pix_stride, src.N * src.H * src.W, src.C,
                                          int(concat.same_grid(idx)), qp.zp, m, s, o.zp, o.qmin,
                                          o.qmax, st)
            elif kind == "gap":
                layer, x, y, area = payload
                m, s = layer.multiplier(area)
                rc = raw.qa_gap16_dev(x.ptr, x.plane, x.pix_stride, x.N, area, x.C, layer.in_zp,
                                      m, s, layer.out_zp, layer.out_qmin, layer.out_qmax, y.ptr,
                                      y.plane, y.pix_stride, st)
            elif kind == "lut":
                layer, x, y, ldev = payload
                rc = raw.qa_lut16_dev(x.ptr, x.plane, x.pix_stride, y.ptr, y.plane, y.pix_stride,
                                      x.N * x.H * x.W, x.C, int(layer.lut_offset),
                                      ldev.data_ptr(), len(layer.lut), st)
            elif kind == "add":
                layer, a, b, y = payload
                (ma, sa), (mb, sb) = layer._mult
                qa, qb = layer.in_qp
                o = layer.out_qp[0]
                rc = raw.qa_add16_dev(a.ptr, a.plane, a.pix_stride, b.ptr, b.plane, b.pix_stride,
                                      y.ptr, y.plane, y.pix_stride, a.N * a.H * a.W, a.C, qa.zp,
                                      ma, sa, qb.zp, mb, sb, layer._sign, o.zp, o.qmin, o.qmax,
                                      st)
            elif kind == "bn":
                layer, x, y, (mdev, sdev, bdev) = payload
                rc = raw.qa_bn16_dev(x.ptr, x.plane, x.pix_stride, y.ptr, y.plane, y.pix_stride,
                                     x.N * x.H * x.W, x.C, layer.in_zp, mdev.data_ptr(),
                                     sdev.data_ptr(), bdev.data_ptr(), layer.out_zp,
                                     layer.out_qmin, layer.out_qmax, st)
            elif kind == "mul":
                layer, a, b, y = payload
                qa, qb = layer.in_qp
                o = layer.out_qp[0]
                rc = raw.qa_mul16_dev(a.ptr, a.plane, a.pix_stride, b.ptr, b.plane, b.pix_stride,
                                      y.ptr, y.plane, y.pix_stride, a.N * a.H * a.W, a.C, qa.zp,
                                      qb.zp, layer._mult, layer._shift, o.zp, o.qmin, o.qmax,
                                      st)
            elif kind == "maxpool":
                layer, x, y = payload
                from quantanything_b200.float_ops import pool_geometry

                k, s_, dl, pd = pool_geometry(layer.node, (x.N, x.C, x.H, x.W))
                rc = raw.qa_maxpool16_dev(x.ptr, x.plane, x.pix_stride, y.ptr, y.plane,
                                          y.pix_stride, x.N, x.H, x.W, x.C, k[0], k[1], s_[0],
                                          s_[1], pd[0], pd[1], dl[0], dl[1], y.H, y.W,
                                          layer.in_qmin, st)
            elif kind == "window":
                # pure data movement: the byte copy on each plane (fill = the
                # zero point's low byte, then its high byte)
                layer, x, y, geom, fill = payload
                rc = 0
                for plane, f in ((0, fill & 0xFF), (1, (fill >> 8) & 0xFF)):
                    if rc == 0:
                        rc = raw.qa_window_copy_bytes_dev(
                            x.ptr + plane * x.plane, y.ptr + plane * y.plane, y.pix_stride, y.N,
                            y.C, y.H, y.W, geom[0].ctypes.data, geom[1].ctypes.data,
                            geom[2].ctypes.data, geom[3].ctypes.data, f, st)
            elif kind == "softmax":
                layer, x = payload
                qi, o = layer.in_qp[0], layer.out_qp[0]
                rc = raw.qa_softmax16_dev(x.ptr, x.plane, x.pix_stride, x.N, x.C,
                                          float(qi.scale), qi.zp, float(o.scale), o.zp, o.qmin,
                                          o.qmax, self.out_q.data_ptr(), self.out_f32.data_ptr(),
                                          float(o.scale), o.zp, st)
            else:
                rc = self._launch_step(kind, payload, raw, st)
            _check(self.lib, rc, f"{kind} step (16-bit)")
            if on_step is not None:
                on_step(n)
            n += 1
        self.launch_count = n
        return n

    # ------------------------------------------------------------ costs --
    def step_costs(self):
        """Algorithmic (bytes, integer ops) per step with 2-byte activations
        and weights: ResidentNet's byte counts doubled, except the float32
        input of the quantize step."""
        costs = []
        for (label, nbytes, ops), (kind, payload) in zip(super().step_costs(), self.steps):
            if kind == "quantize":
                N, C, H, W = self.in_shape
                nbytes = N * C * H * W * 4 + 2 * N * H * W * self._in_view.pix_stride
            else:
                nbytes *= 2
            costs.append((label, nbytes, ops))
        return costs

    def tensor(self, name):
        """A planned tensor as int32 NCHW (inspection helper; copies)."""
        v = self._views[name]
        rows = v.N * v.H * v.W
        lo = torch.as_strided(v.buf, (rows, v.C), (v.pix_stride, 1), v.offset).to(torch.int32)
        hi = torch.as_strided(v.buf, (rows, v.C), (v.pix_stride, 1), v.offset + v.plane)
        t = lo + hi.view(torch.int8).to(torch.int32) * 256 + self._act_shift
        return t.reshape(v.N, v.H, v.W, v.C).permute(0, 3, 1, 2).contiguous()
