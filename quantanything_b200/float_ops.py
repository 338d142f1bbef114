"""Host NumPy operators used around the integer hot path.

Three users, mirroring the reference's ``quantization/float_ops.py``:

* LUT construction: every element-wise unary op a ``FusedElementwise`` node
  may contain is evaluated on the dequantized input grid, in the same float
  arithmetic as the reference, so tables are bit-identical;
* the host (drop-in ABI) execution of scale-preserving layout ops on int32
  tensors -- Split, Slice, Pad (with the zero point), MaxPool (padded with
  qmin), Flatten, Reshape, Transpose, (Un)Squeeze (quant_layers.py:642-650);
* float fallbacks (Softmax, LayerNormalization, activation x activation
  MatMul) and the float forward pass of calibration.

Convolution and GEMM in float mode call the CUDA library
(``native.conv2d_f32`` / ``native.gemm_f32``) like the reference's native
routes (float_ops.py:151-180).
"""

import numpy as np
from numpy.lib.stride_tricks import sliding_window_view

from quantanything_b200 import native

OPS = {}
UNARY_OPS = {}


class UnsupportedOp(NotImplementedError):
    """An operator without an implementation here (float_ops.py:47)."""


def op(*names):
    def deco(fn):
        for n in names:
            OPS[n] = fn
        return fn

    return deco


def unary(name):
    def deco(fn):
        UNARY_OPS[name] = fn
        OPS[name] = lambda node, inputs, opset, **kw: [fn(node, inputs[0])]
        return fn

    return deco


def run_node(node, inputs, opset=13, **kw):
    fn = OPS.get(node.op_type)
    if fn is None:
        raise UnsupportedOp(f"operator '{node.op_type}' (node '{node.name}') is not supported")
    out = fn(node, inputs, opset, **kw)
    return list(out) if isinstance(out, (list, tuple)) else [out]


def normalize_feeds(graph, feeds):
    """Bare array -> {single input name: float32 array} (float_ops.py:88-98)."""
    if not isinstance(feeds, dict):
        names = graph.input_names
        if len(names) != 1:
            raise ValueError(f"model has {len(names)} inputs; pass a dict keyed by {names}")
        feeds = {names[0]: feeds}
    return {k: np.asarray(v, dtype=np.float32) for k, v in feeds.items()}


def run_float(graph, feeds, keep_all=False, lib=None):
    """Float32 forward pass of the whole graph (float_ops.py:63-85)."""
    env = dict(graph.initializers)
    env.update(normalize_feeds(graph, feeds))
    for node in graph.nodes:
        args = [env[i] if i else None for i in node.inputs]
        env.update(zip(node.outputs, run_node(node, args, graph.opset, lib=lib)))
    if keep_all:
        return env
    res = [env[o] for o in graph.outputs]
    return res[0] if len(res) == 1 else res


def _axis(a, ndim):
    return a + ndim if a < 0 else a


def _attr_or_input(node, inputs, idx, name, default=None):
    if len(inputs) > idx and inputs[idx] is not None:
        return np.asarray(inputs[idx]).astype(np.int64).tolist()
    return node.attr(name, default)


def conv_pads(node, in_hw, kernel, strides, dilations):
    """``pads`` / ``auto_pad`` -> (top, left, bottom, right) (float_ops.py:132-148)."""
    auto = node.attr("auto_pad", "NOTSET")
    if auto in ("SAME_UPPER", "SAME_LOWER"):
        pads = []
        for size, k, s, d in zip(in_hw, kernel, strides, dilations):
            out = -(-size // s)
            total = max((out - 1) * s + d * (k - 1) + 1 - size, 0)
            lo, hi = total // 2, total - total // 2
            pads.append((lo, hi) if auto == "SAME_UPPER" else (hi, lo))
        return (pads[0][0], pads[1][0], pads[0][1], pads[1][1])
    if auto == "VALID":
        return (0, 0, 0, 0)
    p = node.attr("pads", [0, 0, 0, 0])
    return (p[0], p[1], p[2], p[3])


# ------------------------------------------------------------- linear ops --
@op("Conv")
def _conv(node, inputs, opset, **kw):
    x, w = inputs[0], inputs[1]
    strides = tuple(node.attr("strides", [1, 1]))
    dil = tuple(node.attr("dilations", [1, 1]))
    pads = conv_pads(node, x.shape[2:], w.shape[2:], strides, dil)
    lib = kw.get("lib") or native.get_library()
    y = lib.conv2d_f32(x, w, strides, pads, dil, node.attr("group", 1))
    if len(inputs) > 2 and inputs[2] is not None:
        y = y + inputs[2].reshape(1, -1, 1, 1)
    return y


@op("BatchNormalization")
def _batchnorm(node, inputs, opset, **kw):
    """Inference BatchNorm (float_ops.py:200-206): x * a + b with
    a = gamma / sqrt(var + eps), b = beta - a * mean, in float32."""
    x, gamma, beta, mean, var = inputs[:5]
    shape = [1, -1] + [1] * (x.ndim - 2)
    a = gamma / np.sqrt(var + node.attr("epsilon", 1e-5))
    b = beta - a * mean
    return (x * a.reshape(shape) + b.reshape(shape)).astype(np.float32)


@op("Gemm")
def _gemm(node, inputs, opset, **kw):
    a, b = inputs[0], inputs[1]
    if node.attr("transA", 0):
        a = a.T
    if node.attr("transB", 0):
        b = b.T
    lib = kw.get("lib") or native.get_library()
    y = np.float32(node.attr("alpha", 1.0)) * lib.gemm_f32(a, b)
    if len(inputs) > 2 and inputs[2] is not None:
        y = y + np.float32(node.attr("beta", 1.0)) * inputs[2]
    return y.astype(np.float32)


@op("MatMul")
def _matmul(node, inputs, opset, **kw):
    y = np.matmul(inputs[0], inputs[1]).astype(np.float32)
    if len(inputs) > 2 and inputs[2] is not None:
        y = y + inputs[2]
    return y


@op("FusedElementwise")
def _fused(node, inputs, opset, **kw):
    """Element-wise chain collected by the reference's fusion pass
    (graph_passes.py:208-272): ``attrs['nodes']`` in order, ``attrs['consts']``."""
    env = dict(node.attrs.get("consts", {}))
    env[node.inputs[0]] = inputs[0]
    for sub in node.attrs["nodes"]:
        args = [env[i] if i else None for i in sub.inputs]
        env[sub.outputs[0]] = run_node(sub, args, opset, **kw)[0]
    return env[node.outputs[0]]


def _binary(fn):
    return lambda node, inputs, opset, **kw: fn(inputs[0], inputs[1])


OPS["Add"] = _binary(np.add)
OPS["Sub"] = _binary(np.subtract)
OPS["Mul"] = _binary(np.multiply)
OPS["Div"] = _binary(np.divide)
OPS["Max"] = _binary(np.maximum)
OPS["Min"] = _binary(np.minimum)


# ---------------------------------------------------- element-wise unary --
# Each formula follows float_ops.py:226-319 of the reference: float64 where
# the reference widens, float32 results.
@unary("Sigmoid")
def _sigmoid(node, x):
    return (1.0 / (1.0 + np.exp(-x.astype(np.float64)))).astype(np.float32)


@unary("Relu")
def _relu(node, x):
    return np.maximum(x, 0)


@unary("LeakyRelu")
def _leaky(node, x):
    return np.where(x >= 0, x, node.attr("alpha", 0.01) * x).astype(np.float32)


@unary("Tanh")
def _tanh(node, x):
    return np.tanh(x).astype(np.float32)


@unary("HardSigmoid")
def _hard_sigmoid(node, x):
    return np.clip(node.attr("alpha", 0.2) * x + node.attr("beta", 0.5), 0, 1).astype(np.float32)


@unary("HardSwish")
def _hard_swish(node, x):
    return (x * np.clip(x / 6.0 + 0.5, 0, 1)).astype(np.float32)


@unary("Elu")
def _elu(node, x):
    a = node.attr("alpha", 1.0)
    return np.where(x > 0, x, a * np.expm1(np.minimum(x, 0))).astype(np.float32)


@unary("Softplus")
def _softplus(node, x):
    return np.logaddexp(0, x.astype(np.float64)).astype(np.float32)


@unary("Abs")
def _abs(node, x):
    return np.abs(x)


@unary("Neg")
def _neg(node, x):
    return -x


@unary("Sqrt")
def _sqrt(node, x):
    return np.sqrt(x).astype(np.float32)


@unary("Exp")
def _exp(node, x):
    return np.exp(x.astype(np.float64)).astype(np.float32)


# Abramowitz & Stegun formula 7.1.26 (|error| < 1.5e-7), the erf the
# reference uses (float_ops.py:289-305): erf(x) = 1 - t*P(t)*exp(-x^2) with
# t = 1 / (1 + p|x|), odd in x.
_AS_P = 0.3275911
_AS_A = (0.254829592, -0.284496736, 1.421413741, -1.453152027, 1.061405429)


def erf_as(x):
    x = x.astype(np.float64)
    ax = np.abs(x)
    t = 1.0 / (1.0 + _AS_P * ax)
    a1, a2, a3, a4, a5 = _AS_A
    poly = t * (a1 + t * (a2 + t * (a3 + t * (a4 + t * a5))))
    return np.sign(x) * (1.0 - poly * np.exp(-ax * ax))


@unary("Erf")
def _erf(node, x):
    return erf_as(x).astype(np.float32)


@unary("Gelu")
def _gelu(node, x):
    x64 = x.astype(np.float64)
    if node.attr("approximate", "none") == "tanh":
        inner = np.sqrt(2 / np.pi) * (x64 + 0.044715 * x64**3)
        return (0.5 * x64 * (1 + np.tanh(inner))).astype(np.float32)
    return (0.5 * x64 * (1 + erf_as(x64 / np.sqrt(2)))).astype(np.float32)


@op("Clip")
def _clip(node, inputs, opset, **kw):
    lo = inputs[1] if len(inputs) > 1 and inputs[1] is not None else node.attr("min")
    hi = inputs[2] if len(inputs) > 2 and inputs[2] is not None else node.attr("max")
    return np.clip(inputs[0], lo, hi)


@op("Pow")
def _pow(node, inputs, opset, **kw):
    return np.power(inputs[0].astype(np.float64),
                    np.asarray(inputs[1]).astype(np.float64)).astype(np.float32)


# --------------------------------------------------------- normalization --
@op("LayerNormalization")
def _layer_norm(node, inputs, opset, **kw):
    """float64 mean / variance over the trailing axes (float_ops.py:336-347)."""
    x = inputs[0].astype(np.float64)
    axis = _axis(node.attr("axis", -1), x.ndim)
    axes = tuple(range(axis, x.ndim))
    mean = x.mean(axis=axes, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=axes, keepdims=True)
    y = (x - mean) / np.sqrt(var + node.attr("epsilon", 1e-5))
    y = y * inputs[1]
    if len(inputs) > 2 and inputs[2] is not None:
        y = y + inputs[2]
    return y.astype(np.float32)


def softmax_axis(node, opset, ndim):
    return _axis(node.attr("axis", -1 if opset >= 13 else 1), ndim)


@op("LogSoftmax")
def _log_softmax(node, inputs, opset, **kw):
    """float64, max-subtracted (float_ops.py:388-395)."""
    x = inputs[0].astype(np.float64)
    axis = softmax_axis(node, opset, x.ndim)
    z = x - x.max(axis=axis, keepdims=True)
    return (z - np.log(np.exp(z).sum(axis=axis, keepdims=True))).astype(np.float32)


@op("ReduceMean")
def _reduce_mean(node, inputs, opset, **kw):
    x = inputs[0]
    axes = _attr_or_input(node, inputs, 1, "axes")
    axes = tuple(_axis(a, x.ndim) for a in axes) if axes is not None and len(axes) else None
    return x.mean(axis=axes, keepdims=bool(node.attr("keepdims", 1))).astype(np.float32)


@op("Softmax")
def _softmax(node, inputs, opset, **kw):
    """float64, max-subtracted (float_ops.py:380-385)."""
    x = inputs[0].astype(np.float64)
    axis = softmax_axis(node, opset, x.ndim)
    e = np.exp(x - x.max(axis=axis, keepdims=True))
    return (e / e.sum(axis=axis, keepdims=True)).astype(np.float32)


# ---------------------------------------------------------------- shapes --
# ONNX TensorProto element types -> NumPy (the ones a Cast can name)
_ONNX_DTYPES = {1: np.float32, 2: np.uint8, 3: np.int8, 4: np.uint16, 5: np.int16, 6: np.int32,
                7: np.int64, 9: np.bool_, 10: np.float16, 11: np.float64, 12: np.uint32,
                13: np.uint64}


@op("Cast")
def _cast(node, inputs, opset, **kw):
    return inputs[0].astype(_ONNX_DTYPES[int(node.attr("to"))])


@op("Shape")
def _shape(node, inputs, opset, **kw):
    shape = np.array(inputs[0].shape, dtype=np.int64)
    return shape[node.attr("start", 0): node.attr("end", None)]


@op("Gather")
def _gather(node, inputs, opset, **kw):
    return np.take(inputs[0], np.asarray(inputs[1]).astype(np.int64), axis=node.attr("axis", 0))


@op("Expand")
def _expand(node, inputs, opset, **kw):
    shape = tuple(int(v) for v in np.asarray(inputs[1]).reshape(-1))
    return np.broadcast_to(inputs[0], np.broadcast_shapes(inputs[0].shape, shape)).copy()


@op("Identity", "Dropout")
def _identity(node, inputs, opset, **kw):
    return inputs[0]


@op("Reshape")
def _reshape(node, inputs, opset, **kw):
    x = inputs[0]
    shape = [int(s) for s in np.asarray(inputs[1]).reshape(-1)]
    if not node.attr("allowzero", 0):
        shape = [x.shape[i] if s == 0 else s for i, s in enumerate(shape)]
    return x.reshape(shape)


@op("Flatten")
def _flatten(node, inputs, opset, **kw):
    x = inputs[0]
    axis = _axis(node.attr("axis", 1), x.ndim)
    return x.reshape(int(np.prod(x.shape[:axis])), -1)


@op("Squeeze")
def _squeeze(node, inputs, opset, **kw):
    axes = _attr_or_input(node, inputs, 1, "axes")
    x = inputs[0]
    if axes is None:
        return np.squeeze(x)
    return np.squeeze(x, axis=tuple(_axis(a, x.ndim) for a in axes))


@op("Unsqueeze")
def _unsqueeze(node, inputs, opset, **kw):
    axes = _attr_or_input(node, inputs, 1, "axes")
    x = inputs[0]
    nd = x.ndim + len(axes)
    for a in sorted(_axis(a, nd) for a in axes):
        x = np.expand_dims(x, a)
    return x


@op("Transpose")
def _transpose(node, inputs, opset, **kw):
    perm = node.attr("perm")
    return np.transpose(inputs[0], perm if perm else None)


@op("Concat")
def _concat(node, inputs, opset, **kw):
    return np.concatenate(inputs, axis=node.attr("axis"))


def split_sizes(node, inputs, dim):
    sizes = _attr_or_input(node, inputs, 1, "split")
    n_out = len(node.outputs)
    return list(sizes) if sizes else [dim // n_out] * n_out


@op("Split")
def _split(node, inputs, opset, **kw):
    x = inputs[0]
    axis = _axis(node.attr("axis", 0), x.ndim)
    sizes = split_sizes(node, inputs, x.shape[axis])
    return list(np.split(x, np.cumsum(sizes)[:-1], axis=axis))


@op("Slice")
def _slice(node, inputs, opset, **kw):
    x = inputs[0]
    starts = _attr_or_input(node, inputs, 1, "starts")
    ends = _attr_or_input(node, inputs, 2, "ends")
    axes = _attr_or_input(node, inputs, 3, "axes", list(range(len(starts))))
    steps = _attr_or_input(node, inputs, 4, "steps", [1] * len(starts))
    index = [slice(None)] * x.ndim
    for s, e, a, st in zip(starts, ends, axes, steps):
        index[_axis(a, x.ndim)] = slice(None if s >= 2**62 else s,
                                        None if abs(e) >= 2**62 else e, st)
    return x[tuple(index)]


@op("Pad")
def _pad(node, inputs, opset, pad_value=None, **kw):
    x = inputs[0]
    pads = _attr_or_input(node, inputs, 1, "pads")
    if pad_value is None:
        if len(inputs) > 2 and inputs[2] is not None:
            pad_value = np.asarray(inputs[2]).reshape(()).item()
        else:
            pad_value = node.attr("value", 0)
    n = x.ndim
    width = [(pads[i], pads[i + n]) for i in range(n)]
    return np.pad(x, width, mode="constant", constant_values=pad_value)


def pool_geometry(node, x_shape):
    """kernel, strides, dilations, (top, left, bottom, right) incl. ceil_mode
    (float_ops.py:517-534)."""
    kernel = tuple(node.attr("kernel_shape"))
    strides = tuple(node.attr("strides", [1] * len(kernel)))
    dil = tuple(node.attr("dilations", [1] * len(kernel)))
    pads = list(conv_pads(node, x_shape[2:], kernel, strides, dil))
    if node.attr("ceil_mode", 0):
        for ax in range(2):
            size = x_shape[2 + ax] + pads[ax] + pads[ax + 2]
            ek = dil[ax] * (kernel[ax] - 1) + 1
            out = -(-(size - ek) // strides[ax]) + 1
            pads[ax + 2] += max((out - 1) * strides[ax] + ek - size, 0)
    return kernel, strides, dil, tuple(pads)


@op("AveragePool")
def _avgpool(node, inputs, opset, **kw):
    """Window mean; padded positions count only with ``count_include_pad``
    (float_ops.py:563-577)."""
    x = inputs[0].astype(np.float32)
    kernel, strides, dil, pads = pool_geometry(node, x.shape)
    spec = ((0, 0), (0, 0), (pads[0], pads[2]), (pads[1], pads[3]))

    def window_sum(t):
        ek = [d * (k - 1) + 1 for k, d in zip(kernel, dil)]
        win = sliding_window_view(np.pad(t, spec), tuple(ek), axis=(2, 3))
        return win[:, :, :: strides[0], :: strides[1], :: dil[0], :: dil[1]].sum(axis=(4, 5))

    total = window_sum(x)
    if node.attr("count_include_pad", 0):
        return (total / (kernel[0] * kernel[1])).astype(np.float32)
    return (total / window_sum(np.ones_like(x[:1, :1]))).astype(np.float32)


@op("MaxPool")
def _maxpool(node, inputs, opset, pad_value=None, **kw):
    x = inputs[0]
    kernel, strides, dil, pads = pool_geometry(node, x.shape)
    if pad_value is None:
        pad_value = -np.inf if np.issubdtype(x.dtype, np.floating) else np.iinfo(x.dtype).min
    xp = np.pad(x, ((0, 0), (0, 0), (pads[0], pads[2]), (pads[1], pads[3])),
                constant_values=pad_value)
    ek = [d * (k - 1) + 1 for k, d in zip(kernel, dil)]
    win = sliding_window_view(xp, tuple(ek), axis=(2, 3))
    win = win[:, :, :: strides[0], :: strides[1], :: dil[0], :: dil[1]]
    return win.max(axis=(4, 5))


@op("GlobalAveragePool")
def _gap(node, inputs, opset, **kw):
    x = inputs[0]
    return x.mean(axis=tuple(range(2, x.ndim)), keepdims=True).astype(np.float32)


@op("GlobalMaxPool")
def _gmp(node, inputs, opset, **kw):
    x = inputs[0]
    return x.max(axis=tuple(range(2, x.ndim)), keepdims=True)
