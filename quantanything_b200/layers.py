"""Quantized layers: calibration, parameter preparation and the integer path.

Mirrors the reference's ``quantization/quant_layers.py`` (same class names,
attributes and integer sequence) so a graph quantized here runs the same
integer arithmetic.  Each layer computes its integer parameters once in
``prepare()`` -- centred weights, integer bias, per-channel fixed-point
multipliers, activation tables -- exactly as the reference does; the
device-resident executor reads those attributes.

Kernel calls go through ``self.lib`` (the container's kernel library: the
CUDA build in production).  The host-side integer path below
(``quantized_infer_integer``) is the drop-in execution model: one library
call per layer on host int32 tensors, as under the reference with QA_LIB
pointing at the CUDA library.
"""

import numpy as np

from quantanything_b200 import native
from quantanything_b200.float_ops import UNARY_OPS, conv_pads, run_node
from quantanything_b200.utils import (
    QParams,
    calculate_scale_zp,
    parse_quant_type,
    quantize_multiplier,
    quantize_multipliers,
)

MAX_LUT_BITS = 16  # quant_layers.py:35


def _min_max(x, lo, hi):
    a, b = float(np.min(x)), float(np.max(x))
    return (a, b) if lo is None else (min(lo, a), max(hi, b))


def _bias_range(num_bits):
    """int32 range for <= 8-bit models, int64 beyond (quant_layers.py:46-47)."""
    return (-(2**63), 2**63 - 1) if num_bits > 8 else (-(2**31), 2**31 - 1)


def _np_quantize(x, scale, zp, qmin, qmax):
    """Per-channel host quantization, half to even (utils.py:110-114)."""
    scale = np.asarray(scale, dtype=np.float64)
    safe = np.where(scale == 0, 1.0, scale)
    q = np.round(np.asarray(x).astype(np.float64) / safe) + zp
    q = np.where(scale == 0, zp, q)
    return np.clip(q, qmin, qmax).astype(np.int32 if qmax < 2**31 else np.int64)


def _weight_qparams(w, axis, quant_type, per_channel):
    """Per-slice (scale, zp) along ``axis`` (quant_layers.py:50-67)."""
    flat = np.moveaxis(w, axis, 0).reshape(w.shape[axis], -1)
    if per_channel:
        params = [calculate_scale_zp(r.min(), r.max(), quant_type)[:2] for r in flat]
    else:
        params = [calculate_scale_zp(flat.min(), flat.max(), quant_type)[:2]] * flat.shape[0]
    return (np.array([p[0] for p in params], dtype=np.float64),
            np.array([p[1] for p in params], dtype=np.int64))


class BaseQuantLayer:
    """One graph node; integer fallback = dequantize -> float op -> quantize
    (quant_layers.py:70-205)."""

    def __init__(self, node, graph, quant_type="int8", per_channel=True, lib=None):
        self.node, self.graph, self.name = node, graph, node.name
        self.quant_type, self.per_channel = quant_type, per_channel
        self.num_bits, self.signed = parse_quant_type(quant_type)
        self._lib = lib
        self.data_inputs = self._select_data_inputs()
        self.out_min = [None] * len(node.outputs)
        self.out_max = [None] * len(node.outputs)
        self.in_qp, self.out_qp = [], []

    @property
    def lib(self):
        return self._lib if self._lib is not None else native.get_library()

    def _select_data_inputs(self):
        return [i for i in self.node.inputs if i and not self.graph.is_constant(i)]

    in_scale = property(lambda s: s.in_qp[0].scale if s.in_qp else None)
    in_zp = property(lambda s: s.in_qp[0].zp if s.in_qp else None)
    in_qmin = property(lambda s: s.in_qp[0].qmin if s.in_qp else None)
    in_qmax = property(lambda s: s.in_qp[0].qmax if s.in_qp else None)
    out_scale = property(lambda s: s.out_qp[0].scale if s.out_qp else None)
    out_zp = property(lambda s: s.out_qp[0].zp if s.out_qp else None)
    out_qmin = property(lambda s: s.out_qp[0].qmin if s.out_qp else None)
    out_qmax = property(lambda s: s.out_qp[0].qmax if s.out_qp else None)

    # ---------------------------------------------------------------- float --
    def _full_args(self, data_args):
        data = dict(zip(self.data_inputs, data_args))
        return [None if not n else data[n] if n in data else self.graph.initializers[n]
                for n in self.node.inputs]

    def _run_float(self, data_args, **kw):
        return run_node(self.node, self._full_args(data_args), self.graph.opset, lib=self.lib,
                        **kw)

    def calibrate(self, inputs):
        outs = self._run_float(inputs)
        for i, o in enumerate(outs):
            self.out_min[i], self.out_max[i] = _min_max(o, self.out_min[i], self.out_max[i])
        return outs

    # ------------------------------------------------------------- finalize --
    def _default_out_qparams(self):
        qps = []
        for i, name in enumerate(self.node.outputs):
            if self.out_min[i] is None:
                raise ValueError(f"Layer {self.name}: output '{name}' was never observed; "
                                 "run calibrate() before finalizing")
            qps.append(QParams(*calculate_scale_zp(self.out_min[i], self.out_max[i],
                                                   self.quant_type)))
        return qps

    def finalize_calibration(self, container):
        self.in_qp = [container.qparams[n] for n in self.data_inputs]
        self.out_qp = self._default_out_qparams()
        for name, qp in zip(self.node.outputs, self.out_qp):
            container.qparams[name] = qp
        self.prepare()

    def load_qparams(self, container):
        self.in_qp = [container.qparams[n] for n in self.data_inputs]
        self.out_qp = [container.qparams[n] for n in self.node.outputs]
        self.prepare()

    def prepare(self):
        """Integer parameters from the in/out qparams."""

    def _check_ready(self):
        if not self.out_qp or (self.data_inputs and not self.in_qp):
            raise ValueError(f"Layer {self.name} is not calibrated.")

    # -------------------------------------------------------------- integer --
    def quantized_infer_integer(self, inputs):
        self._check_ready()
        xs = [self.lib.dequantize_f32(v, qp.scale, qp.zp) for v, qp in zip(inputs, self.in_qp)]
        outs = self._run_float(xs)
        return [self.lib.quantize_f32(o, qp.scale, qp.zp, qp.qmin, qp.qmax)
                for o, qp in zip(outs, self.out_qp)]


class _WeightedLayer(BaseQuantLayer):
    """Shared weight / bias quantization of Conv and Gemm (quant_layers.py:209-287)."""

    weight_axis = 0

    def __init__(self, *args, **kw):
        super().__init__(*args, **kw)
        bits, signed = self.num_bits, self.signed
        self.w_qmin, self.w_qmax = ((-(1 << (bits - 1)), (1 << (bits - 1)) - 1) if signed
                                    else (0, (1 << bits) - 1))
        self.b_qmin, self.b_qmax = _bias_range(bits)
        self.bias_int = None

    def _select_data_inputs(self):
        return [self.node.inputs[0]]

    def _weights(self):
        raise NotImplementedError

    def prepare(self):
        w, bias = self._weights()
        scale_c, zp_c = _weight_qparams(w, self.weight_axis, self.quant_type, self.per_channel)
        bshape = [1] * w.ndim
        bshape[self.weight_axis] = -1
        if self.per_channel:
            self.w_scale, self.w_zp = scale_c, zp_c
        else:
            self.w_scale, self.w_zp = float(scale_c[0]), int(zp_c[0])
        self._w_zp_c = zp_c
        self._reduction = int(np.prod(w.shape) // w.shape[self.weight_axis])
        self.wide = native.accumulator_is_wide(self.num_bits, self._reduction)
        self.w_q = _np_quantize(w, scale_c.reshape(bshape), zp_c.reshape(bshape),
                                self.w_qmin, self.w_qmax)
        self.w_centered = (self.w_q.astype(np.int64) - zp_c.reshape(bshape)).astype(
            np.int32 if self.wide else np.int16)
        if bias is not None:
            self.bias_int = np.clip(np.round(bias / (self.in_scale * scale_c)),
                                    self.b_qmin, self.b_qmax).astype(np.int64)
        else:
            self.bias_int = None
        self.q_mult, self.shift = quantize_multipliers(self.in_scale * scale_c / self.out_scale)
        if not self.per_channel:
            self.q_mult, self.shift = self.q_mult[:1], self.shift[:1]


class ConvQuantize(_WeightedLayer):
    """2-D convolution with constant weights (quant_layers.py:290-341)."""

    def _weights(self):
        w = self.graph.initializers[self.node.inputs[1]].astype(np.float32)
        bias = None
        if len(self.node.inputs) > 2 and self.node.inputs[2]:
            bias = self.graph.initializers[self.node.inputs[2]].astype(np.float32)
        return w, bias

    def geometry(self, x_shape):
        strides = tuple(self.node.attr("strides", [1, 1]))
        dil = tuple(self.node.attr("dilations", [1, 1]))
        pads = conv_pads(self.node, x_shape[2:], self.w_q.shape[2:], strides, dil)
        return strides, pads, dil, self.node.attr("group", 1)

    def quantized_infer_integer(self, inputs):
        self._check_ready()
        x = np.asarray(inputs[0])
        strides, pads, dil, groups = self.geometry(x.shape)
        acc = self.lib.conv2d_int(x - self.in_zp, self.w_centered, strides, pads, dil, groups,
                                  self.wide)
        n, cout, oh, ow = acc.shape
        return [self.lib.requantize(acc, n, cout, oh * ow, self.q_mult, self.shift,
                                    self.out_zp, self.out_qmin, self.out_qmax,
                                    pre_bias=self.bias_int)]


class GemmQuantize(_WeightedLayer):
    """Gemm / MatMul against a constant [K, N] weight (quant_layers.py:344-402)."""

    weight_axis = 1

    def _weights(self):
        node = self.node
        b = self.graph.initializers[node.inputs[1]].astype(np.float32)
        bias = None
        if node.op_type == "Gemm":
            if node.attr("transB", 0):
                b = b.T
            b = b * np.float32(node.attr("alpha", 1.0))
            if len(node.inputs) > 2 and node.inputs[2]:
                c = self.graph.initializers[node.inputs[2]].astype(np.float32)
                bias = np.broadcast_to(c.reshape(-1), (b.shape[1],)).astype(np.float32)
                bias = bias * np.float32(node.attr("beta", 1.0))
        elif len(node.inputs) > 2 and node.inputs[2]:
            bias = np.ascontiguousarray(
                self.graph.initializers[node.inputs[2]].astype(np.float32).reshape(-1))
        return np.ascontiguousarray(b), bias

    def out_shape(self, x_shape):
        if self.node.op_type == "Gemm":
            return (x_shape[0], self.w_q.shape[1])
        return tuple(x_shape[:-1]) + (self.w_q.shape[1],)

    def quantized_infer_integer(self, inputs):
        self._check_ready()
        x = np.asarray(inputs[0])
        x2 = x.reshape(-1, x.shape[-1]) - self.in_zp
        acc = self.lib.gemm_int(x2, self.w_centered, self.wide)
        m, n = acc.shape
        out = self.lib.requantize(acc, m, n, 1, self.q_mult, self.shift, self.out_zp,
                                  self.out_qmin, self.out_qmax, pre_bias=self.bias_int)
        return [out.reshape(self.out_shape(x.shape))]


class BatchNormalizationQuantize(BaseQuantLayer):
    """Inference BatchNorm as a per-channel integer affine map (quant_layers.py:405-441)."""

    def _select_data_inputs(self):
        return [self.node.inputs[0]]

    def prepare(self):
        gamma, beta, mean, var = (self.graph.initializers[n].astype(np.float64)
                                  for n in self.node.inputs[1:5])
        a = gamma / np.sqrt(var + self.node.attr("epsilon", 1e-5))
        self.A, self.B = a, beta - a * mean
        self.q_mult, self.shift = quantize_multipliers(self.in_scale * a / self.out_scale)
        self.q_B = np.round(self.B / self.out_scale).astype(np.int64)

    def quantized_infer_integer(self, inputs):
        self._check_ready()
        x = np.asarray(inputs[0])
        centred = (x - self.in_zp).astype(np.int32)
        out = self.lib.requantize(centred, x.shape[0], x.shape[1],
                                  int(np.prod(x.shape[2:], dtype=np.int64)), self.q_mult,
                                  self.shift, self.out_zp, self.out_qmin, self.out_qmax,
                                  post_bias=self.q_B)
        return [out.reshape(x.shape)]


class ActivationQuantize(BaseQuantLayer):
    """Element-wise unary function as an integer lookup table (quant_layers.py:445-472)."""

    def _select_data_inputs(self):
        return [self.node.inputs[0]]

    @staticmethod
    def supports(node, graph, quant_type):
        if parse_quant_type(quant_type)[0] > MAX_LUT_BITS:
            return False
        if node.op_type == "Clip":
            return all(graph.is_constant(i) for i in node.inputs[1:] if i)
        return node.op_type in UNARY_OPS or node.op_type == "FusedElementwise"

    def prepare(self):
        qp, o = self.in_qp[0], self.out_qp[0]
        grid = np.arange(qp.qmin, qp.qmax + 1, dtype=np.int64).astype(np.int32)
        x = self.lib.dequantize_f32(grid, qp.scale, qp.zp)
        y = self._run_float([x])[0]
        self.lut = self._quantize_table(y, o)
        self.lut_offset = qp.qmin

    def _quantize_table(self, y, o):
        if o.scale == 0:
            return np.full(y.shape, o.zp, dtype=np.int32)
        y = np.asarray(y)
        if y.dtype in (np.float32, np.float64):
            return self.lib.quantize_f32(y, o.scale, o.zp, o.qmin, o.qmax).astype(np.int32)
        return _np_quantize(y, o.scale, o.zp, o.qmin, o.qmax).astype(np.int32)

    def quantized_infer_integer(self, inputs):
        self._check_ready()
        return [self.lib.lut(np.asarray(inputs[0]), self.lut, self.lut_offset)]


class _MultiInputLayer(BaseQuantLayer):
    def _select_data_inputs(self):
        return [i for i in self.node.inputs if i]

    def _mults(self, in_scales):
        return [quantize_multiplier(s / self.out_scale) for s in in_scales]


class AddQuantize(_MultiInputLayer):
    """Add / Sub with both operands rescaled to the output grid (quant_layers.py:486-513)."""

    def prepare(self):
        self._mult = self._mults([qp.scale for qp in self.in_qp])
        self._sign = -1 if self.node.op_type == "Sub" else 1

    def quantized_infer_integer(self, inputs):
        self._check_ready()
        (ma, sa), (mb, sb) = self._mult
        a, b = self.in_qp
        o = self.out_qp[0]
        return [self.lib.add(inputs[0], inputs[1], a.zp, ma, sa, b.zp, mb, sb, o.zp, o.qmin,
                             o.qmax, self._sign)]


class MulQuantize(_MultiInputLayer):
    """(q1 - z1)(q2 - z2) with one requantize (quant_layers.py:516-540)."""

    def prepare(self):
        self._mult, self._shift = quantize_multiplier(
            self.in_qp[0].scale * self.in_qp[1].scale / self.out_scale)

    def quantized_infer_integer(self, inputs):
        self._check_ready()
        a, b = self.in_qp
        o = self.out_qp[0]
        return [self.lib.mul(inputs[0], inputs[1], a.zp, b.zp, self._mult, self._shift, o.zp,
                             o.qmin, o.qmax)]


class ConcatQuantize(_MultiInputLayer):
    """Rescale each input to the output grid, then concatenate (quant_layers.py:543-560)."""

    def prepare(self):
        self._mult = self._mults([qp.scale for qp in self.in_qp])

    def same_grid(self, i):
        qp, o = self.in_qp[i], self.out_qp[0]
        return qp.scale == o.scale and qp.zp == o.zp

    def quantized_infer_integer(self, inputs):
        self._check_ready()
        o = self.out_qp[0]
        parts = []
        for i, (x, qp, (m, s)) in enumerate(zip(inputs, self.in_qp, self._mult)):
            if self.same_grid(i):
                parts.append(np.clip(x, o.qmin, o.qmax).astype(np.int32))
            else:
                parts.append(self.lib.rescale(x, qp.zp, m, s, o.zp, o.qmin, o.qmax))
        return [np.concatenate(parts, axis=self.node.attr("axis"))]


class GlobalAveragePoolQuantize(BaseQuantLayer):
    """Spatial mean: int64 sum, 1/area folded into the multiplier (quant_layers.py:563-590)."""

    def _select_data_inputs(self):
        return [self.node.inputs[0]]

    def multiplier(self, area):
        """(M0, shift) of in_scale / (out_scale * area), computed per call like
        the reference (quant_layers.py:575-577)."""
        return quantize_multiplier(self.in_scale / (self.out_scale * area))

    def quantized_infer_integer(self, inputs):
        self._check_ready()
        x = np.asarray(inputs[0])
        area = int(np.prod(x.shape[2:]))
        acc = (x.astype(np.int64) - self.in_zp).sum(axis=tuple(range(2, x.ndim)), keepdims=True)
        mult, shift = self.multiplier(area)
        n, c = x.shape[:2]
        return [self.lib.requantize(acc, n, c, 1, mult, shift, self.out_zp, self.out_qmin,
                                    self.out_qmax)]


class ShapingQuantize(BaseQuantLayer):
    """Scale-preserving layout / selection ops on integers (quant_layers.py:593-650)."""

    SUPPORTED = {"Reshape", "Flatten", "Squeeze", "Unsqueeze", "Transpose", "Split", "Slice",
                 "Pad", "MaxPool", "GlobalMaxPool"}

    def _select_data_inputs(self):
        return [self.node.inputs[0]]

    @classmethod
    def supports(cls, node, graph):
        if node.op_type not in cls.SUPPORTED:
            return False
        if not all(graph.is_constant(i) for i in node.inputs[1:] if i):
            return False
        if node.op_type == "Pad":
            if node.attr("mode", "constant") != "constant":
                return False
            value = (graph.initializers[node.inputs[2]] if len(node.inputs) > 2 and node.inputs[2]
                     else node.attr("value", 0))
            return float(np.asarray(value)) == 0.0
        return True

    def _default_out_qparams(self):
        return [self.in_qp[0]] * len(self.node.outputs)

    def quantized_infer_integer(self, inputs):
        self._check_ready()
        kw = {}
        if self.node.op_type == "Pad":
            kw["pad_value"] = self.in_zp
        elif self.node.op_type == "MaxPool":
            kw["pad_value"] = self.in_qmin
        outs = self._run_float([np.asarray(inputs[0])], **kw)
        return [np.ascontiguousarray(o, dtype=np.int32) for o in outs]


def map_node_to_quant(node, graph, quant_type="int8", per_channel=True, lib=None):
    """Layer class for a node (quant_layers.py:653-691)."""
    op_type, const = node.op_type, graph.is_constant
    args = (node, graph, quant_type, per_channel)
    kw = {"lib": lib}
    if op_type == "Conv" and len(node.inputs) > 1 and const(node.inputs[1]):
        w = graph.initializers[node.inputs[1]]
        bias_ok = len(node.inputs) < 3 or not node.inputs[2] or const(node.inputs[2])
        if w.ndim == 4 and bias_ok:
            return ConvQuantize(*args, **kw)
    if op_type in ("Gemm", "MatMul") and len(node.inputs) > 1 and const(node.inputs[1]):
        b = graph.initializers[node.inputs[1]]
        ok = b.ndim == 2 and not (op_type == "Gemm" and node.attr("transA", 0))
        if len(node.inputs) > 2 and node.inputs[2]:
            ok = ok and const(node.inputs[2])
        if ok and not const(node.inputs[0]):
            return GemmQuantize(*args, **kw)
    if op_type == "BatchNormalization" and all(const(i) for i in node.inputs[1:5]):
        return BatchNormalizationQuantize(*args, **kw)
    if ActivationQuantize.supports(node, graph, quant_type):
        return ActivationQuantize(*args, **kw)
    if op_type in ("Add", "Sub") and not all(const(i) for i in node.inputs):
        return AddQuantize(*args, **kw)
    if op_type == "Mul" and not all(const(i) for i in node.inputs):
        return MulQuantize(*args, **kw)
    if op_type == "Concat":
        return ConcatQuantize(*args, **kw)
    if op_type == "GlobalAveragePool":
        return GlobalAveragePoolQuantize(*args, **kw)
    if ShapingQuantize.supports(node, graph):
        return ShapingQuantize(*args, **kw)
    return BaseQuantLayer(*args, **kw)
