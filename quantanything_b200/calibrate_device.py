"""Calibration on the GPU: the float pass and the range reductions.

The reference calibrates by running the float graph batch by batch and
recording min / max of every graph input (quant_container.py:141-149) and
of every layer output (quant_layers.py:130-137).  ``DeviceCalibrator`` runs
the same float graph with every tensor in device memory, one kernel of
the CUDA library per operator (csrc/qa_calibrate.cu; convolutions use the
same CUDA-core kernel as ``qa_conv_f32``), and each kernel folds the values
it writes into the tensor's range slot on the device.  Nothing comes back
to the host until ``ranges()`` copies the whole range table (two float32
words per tensor) once; across GPUs ``allreduce`` combines the tables on
the device with one NCCL all-reduce first.

The float arithmetic follows ``float_ops`` (float32 tensors; float64 where
the reference widens: Sigmoid, Exp, Softplus, Erf / Gelu, Pow, Softmax,
LayerNormalization).  Sums run in another order than NumPy's, so ranges can
differ at the last float32 bit -- the resulting qparams are compared with
the reference's q.json with the same tolerance as the host calibration.

Operators: Conv, Gemm, MatMul, BatchNormalization, the element-wise unary
and binary ops (with NumPy broadcasting), FusedElementwise chains,
LayerNormalization, Softmax (last axis), MaxPool, GlobalAveragePool and the
layout ops (Reshape, Flatten, (Un)Squeeze, Identity, Transpose, Slice,
Split, Concat, Pad, Expand, Gather with constant indices).  Anything else
raises ``UnsupportedGraph``; there is no host fallback.
"""

import ctypes

import numpy as np
import torch

from quantanything_b200 import float_ops
from quantanything_b200.float_ops import conv_pads, pool_geometry, softmax_axis

_P, _I64, _I32, _F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float
_SIGNATURES = {
    "qa_f32_map_dev": [_P, _P, _I64, _I32, _F, _F, _P, _P],
    "qa_f32_binary_dev": [_P, _P, _P, _I32, _P, _P, _P, _I32, _P, _P],
    "qa_f32_copy_dev": [_P, _P, _I32, _P, _P, _P, _P, _P],
    "qa_f32_fill_dev": [_P, _I64, _F, _P, _P],
    "qa_f32_range_dev": [_P, _I64, _P, _P],
    "qa_f32_range_decode_dev": [_P, _P, _I64, _P],
    "qa_f32_gemm_dev": [_P, _P, _P] + [_I64] * 10 + [_F, _P, _P],
    "qa_f32_conv_dev": [_P, _P, _P] + [_I64] * 16 + [_P],
    "qa_f32_softmax_dev": [_P, _P, _I64, _I64, _P, _P],
    "qa_f32_layernorm_dev": [_P, _P, _P, _P, _I64, _I64, ctypes.c_double, _P, _P],
    "qa_f32_maxpool_dev": [_P, _P] + [_I64] * 13 + [_P, _P],
    "qa_f32_plane_mean_dev": [_P, _P, _I64, _I64, _P, _P],
}

MAP_OPS = {"Identity": 0, "Dropout": 0, "Sigmoid": 1, "Relu": 2, "LeakyRelu": 3, "Tanh": 4,
           "HardSigmoid": 5, "HardSwish": 6, "Elu": 7, "Softplus": 8, "Abs": 9, "Neg": 10,
           "Sqrt": 11, "Exp": 12, "Erf": 13}
GELU_ERF, GELU_TANH, CLIP = 14, 15, 16
BINARY_OPS = {"Add": 0, "Sub": 1, "Mul": 2, "Div": 3, "Max": 4, "Min": 5, "Pow": 6}
VIEW_OPS = ("Reshape", "Flatten", "Squeeze", "Unsqueeze", "Transpose", "Slice", "Split")
MAX_RANK = 6


class UnsupportedGraph(NotImplementedError):
    """The graph holds an operator the device calibration does not run."""


def calib_api(lib):
    """Declares the float-pass entry points on a loaded KernelLibrary."""
    raw = lib.raw
    if not getattr(raw, "_qa_calib_declared", False):
        for name, args in _SIGNATURES.items():
            fn = getattr(raw, name)
            fn.restype, fn.argtypes = ctypes.c_int, args
        raw._qa_calib_declared = True
    return raw


def _i64(values):
    return (ctypes.c_int64 * max(len(values), 1))(*[int(v) for v in values])


def _dense_strides(shape):
    out, acc = [], 1
    for d in reversed(shape):
        out.append(acc)
        acc *= int(d)
    return list(reversed(out))


def _broadcast_strides(shape, out_shape):
    """Element strides of a dense ``shape`` read at every index of ``out_shape``."""
    shape = (1,) * (len(out_shape) - len(shape)) + tuple(shape)
    dense = _dense_strides(shape)
    return [0 if s == 1 and o != 1 else st for s, o, st in zip(shape, out_shape, dense)]


def _fold_dims(shape, *strides):
    """Merges adjacent dimensions that every stride list walks contiguously,
    so tensors of any rank fit the kernels' six dimensions when they can."""
    dims = [[int(shape[d])] + [int(s[d]) for s in strides] for d in range(len(shape))
            if shape[d] != 1]
    out = []
    for d in dims:
        if out and all(out[-1][k + 1] == d[k + 1] * d[0] for k in range(len(strides))):
            out[-1][0] *= d[0]
            for k in range(len(strides)):
                out[-1][k + 1] = d[k + 1]
        else:
            out.append(d)
    if not out:
        out = [[1] + [0] * len(strides)]
    return [o[0] for o in out], [[o[k + 1] for o in out] for k in range(len(strides))]


class DeviceCalibrator:
    """Observes calibration batches on the GPU for ``container`` (not yet
    finalized); ``ranges()`` returns ``{key: (lo, hi)}`` with the keys of
    ``QuantContainer.get_ranges``."""

    def __init__(self, container, device=None, lib=None):
        self.c = container
        self.graph = container.graph
        self.lib = lib if lib is not None else container.lib
        self.raw = calib_api(self.lib)
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.keys = [f"in:{t.name}" for t in self.graph.inputs]
        for layer in container.layers:
            self.keys += [f"{layer.name}:{i}" for i in range(len(layer.node.outputs))]
        self.slot = {k: i for i, k in enumerate(self.keys)}
        self.table = torch.empty((len(self.keys), 2), dtype=torch.int32, device=self.device)
        self.table[:, 0] = -1  # min key 0xFFFFFFFF: nothing observed
        self.table[:, 1] = 0
        self._consts = {}
        self.launches = 0

    # ------------------------------------------------------------ helpers --
    @property
    def _st(self):
        if self.device.type != "cuda":
            return None
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _range_ptr(self, key):
        if key is None:
            return None
        return self.table.data_ptr() + 8 * self.slot[key]

    def _call(self, name, *args):
        rc = getattr(self.raw, name)(*args, self._st)
        self.launches += 1
        if rc != 0:
            msg = self.raw.qa_last_error().decode(errors="replace")
            self.raw.qa_clear_error()
            raise RuntimeError(f"{name}: {msg}")

    def _empty(self, shape):
        return torch.empty(tuple(int(s) for s in shape), dtype=torch.float32, device=self.device)

    def _const(self, name, value):
        t = self._consts.get(name)
        if t is None:
            t = torch.from_numpy(np.array(value, dtype=np.float32, order="C")).to(self.device)
            self._consts[name] = t
        return t

    def _dev(self, v, name=None):
        """A computed tensor as is; a constant uploaded (cached by ``name``)."""
        if isinstance(v, torch.Tensor):
            return v
        if name is None:
            return torch.from_numpy(np.array(v, dtype=np.float32, order="C")).to(self.device)
        return self._const(name, v)

    def _range_of(self, t, key):
        if key is not None and t.numel():
            self._call("qa_f32_range_dev", t.data_ptr(), t.numel(), self._range_ptr(key))

    def _copy(self, x, y, shape, xs, ys, x_off=0, y_off=0, key=None):
        shape, (xs, ys) = _fold_dims(shape, xs, ys)
        if len(shape) > MAX_RANK:
            raise UnsupportedGraph(f"copy of rank {len(shape)} beyond {MAX_RANK}")
        self._call("qa_f32_copy_dev", x.data_ptr() + 4 * x_off, y.data_ptr() + 4 * y_off,
                   len(shape), _i64(shape), _i64(xs), _i64(ys), self._range_ptr(key))

    def _binary(self, op, a, b, key, out=None):
        shape = tuple(np.broadcast_shapes(tuple(a.shape), tuple(b.shape)))
        y = out if out is not None else self._empty(shape)
        sa, sb = _broadcast_strides(a.shape, shape), _broadcast_strides(b.shape, shape)
        dims, (sa, sb) = _fold_dims(shape, sa, sb)
        if len(dims) > MAX_RANK:
            raise UnsupportedGraph(f"broadcast of rank {len(dims)} beyond {MAX_RANK}")
        self._call("qa_f32_binary_dev", a.data_ptr(), b.data_ptr(), y.data_ptr(), len(dims),
                   _i64(dims), _i64(sa), _i64(sb), BINARY_OPS[op], self._range_ptr(key))
        return y

    def _map(self, code, x, key, p0=0.0, p1=0.0):
        y = self._empty(x.shape)
        self._call("qa_f32_map_dev", x.data_ptr(), y.data_ptr(), x.numel(), code, p0, p1,
                   self._range_ptr(key))
        return y

    # ------------------------------------------------------------ running --
    def observe(self, x):
        """Runs one calibration batch (array, or dict keyed by input name)
        through the float graph on the device, folding every range."""
        feeds = float_ops.normalize_feeds(self.graph, x)
        env = {}
        for name, value in feeds.items():
            t = torch.from_numpy(np.ascontiguousarray(value, dtype=np.float32)).to(
                self.device, non_blocking=False)
            self._range_of(t, f"in:{name}")
            env[name] = t
        last_use = {}
        for idx, node in enumerate(self.graph.nodes):
            for n in node.inputs:
                last_use[n] = idx
        keep = set(self.graph.outputs)
        for idx, node in enumerate(self.graph.nodes):
            layer = self.c.quant_layers[node.name]
            args = [None if not n else env[n] if n in env else self.graph.initializers[n]
                    for n in node.inputs]
            keys = [f"{layer.name}:{i}" for i in range(len(node.outputs))]
            outs = self._run(node, args, keys)
            env.update(zip(node.outputs, outs))
            for n in set(node.inputs):
                if last_use.get(n) == idx and n not in keep:
                    env.pop(n, None)
        return [env[n] for n in self.graph.outputs]

    def _run(self, node, args, keys):
        op = node.op_type
        names = list(node.inputs)
        if op == "Conv":
            return [self._conv(node, args, names, keys[0])]
        if op == "Gemm":
            return [self._gemm(node, args, names, keys[0])]
        if op == "MatMul":
            return [self._matmul(args, names, keys[0])]
        if op in BINARY_OPS:
            a, b = self._dev(args[0], names[0]), self._dev(args[1], names[1])
            return [self._binary(op, a, b, keys[0])]
        if op == "FusedElementwise":
            return [self._fused(node, args[0], keys[0])]
        if op in MAP_OPS or op in ("Gelu", "Clip"):
            return [self._unary(node, args, keys[0])]
        if op == "BatchNormalization":
            return [self._batchnorm(node, args, keys[0])]
        if op == "LayerNormalization":
            return [self._layernorm(node, args, names, keys[0])]
        if op == "Softmax":
            return [self._softmax(node, args[0], keys[0])]
        if op == "MaxPool":
            return [self._maxpool(node, args[0], keys[0])]
        if op == "GlobalAveragePool":
            return [self._gap(args[0], keys[0])]
        if op in VIEW_OPS:
            return self._layout(node, args, keys)
        if op == "Concat":
            return [self._concat(node, args, names, keys[0])]
        if op == "Pad":
            return [self._pad(node, args, keys[0])]
        if op == "Expand":
            return [self._expand(args, keys[0])]
        if op == "Gather":
            return [self._gather(node, args, keys[0])]
        raise UnsupportedGraph(f"operator '{op}' (node '{node.name}') has no device float kernel")

    # ------------------------------------------------------------ operators --
    def _conv(self, node, args, names, key):
        x, w = args[0], args[1]
        if not isinstance(x, torch.Tensor):
            raise UnsupportedGraph("Conv of a constant input")
        wd = self._dev(w, names[1])
        strides = tuple(node.attr("strides", [1, 1]))
        dil = tuple(node.attr("dilations", [1, 1]))
        N, C, H, W = x.shape
        cout, _, kh, kw = wd.shape
        pt, pl, pb, pr = conv_pads(node, (H, W), (kh, kw), strides, dil)
        oh = (H + pt + pb - dil[0] * (kh - 1) - 1) // strides[0] + 1
        ow = (W + pl + pr - dil[1] * (kw - 1) - 1) // strides[1] + 1
        y = self._empty((N, cout, oh, ow))
        self._call("qa_f32_conv_dev", x.data_ptr(), wd.data_ptr(), y.data_ptr(), N, C, H, W,
                   cout, kh, kw, strides[0], strides[1], pt, pl, dil[0], dil[1],
                   node.attr("group", 1), oh, ow)
        if len(args) > 2 and args[2] is not None:
            b = self._dev(args[2], names[2]).reshape(1, -1, 1, 1)
            return self._binary("Add", y, b, key, out=y)
        self._range_of(y, key)
        return y

    def _gemm_call(self, a, b, batch, M, N, K, sa, sb, alpha, key):
        y = self._empty((batch, M, N))
        self._call("qa_f32_gemm_dev", a.data_ptr(), b.data_ptr(), y.data_ptr(), batch, M, N, K,
                   sa[0], sa[1], sa[2], sb[0], sb[1], sb[2], float(alpha), self._range_ptr(key))
        return y

    def _gemm(self, node, args, names, key):
        a, b = self._dev(args[0], names[0]), self._dev(args[1], names[1])
        ta, tb = node.attr("transA", 0), node.attr("transB", 0)
        M, K = (a.shape[1], a.shape[0]) if ta else (a.shape[0], a.shape[1])
        N = b.shape[0] if tb else b.shape[1]
        sa = (0, 1, M) if ta else (0, K, 1)
        sb = (0, 1, K) if tb else (0, N, 1)
        bias = args[2] if len(args) > 2 else None
        alpha = np.float32(node.attr("alpha", 1.0))
        y = self._gemm_call(a, b, 1, M, N, K, sa, sb, alpha, None if bias is not None else key)
        y = y.reshape(M, N)
        if bias is not None:
            beta = np.float32(node.attr("beta", 1.0))
            c = bias if isinstance(bias, torch.Tensor) else self._const(
                (names[2], float(beta)), beta * np.asarray(bias, dtype=np.float32))
            if isinstance(bias, torch.Tensor) and beta != 1:
                raise UnsupportedGraph("Gemm with beta != 1 on a computed C")
            return self._binary("Add", y, c, key, out=y)
        return y

    def _matmul(self, args, names, key):
        a, b = self._dev(args[0], names[0]), self._dev(args[1], names[1])
        if a.dim() < 2 or b.dim() < 2:
            raise UnsupportedGraph("MatMul of a vector")
        M, K = a.shape[-2], a.shape[-1]
        N = b.shape[-1]
        batch_shape = tuple(np.broadcast_shapes(tuple(a.shape[:-2]), tuple(b.shape[:-2])))
        batch = int(np.prod(batch_shape)) if batch_shape else 1

        def batch_stride(t, mat):
            own = tuple(t.shape[:-2])
            if (int(np.prod(own)) if own else 1) == 1:
                return 0
            if (1,) * (len(batch_shape) - len(own)) + own != batch_shape:
                raise UnsupportedGraph("MatMul with a partially broadcast batch")
            return mat

        if b.dim() == 2 and a.dim() > 2:  # fold the batch into the rows
            y = self._gemm_call(a, b, 1, batch * M, N, K, (0, K, 1), (0, N, 1), 1.0,
                                key if len(args) < 3 or args[2] is None else None)
        else:
            y = self._gemm_call(a, b, batch, M, N, K, (batch_stride(a, M * K), K, 1),
                                (batch_stride(b, K * N), N, 1), 1.0,
                                key if len(args) < 3 or args[2] is None else None)
        y = y.reshape(*batch_shape, M, N)
        if len(args) > 2 and args[2] is not None:
            return self._binary("Add", y, self._dev(args[2], names[2]), key)
        return y

    def _unary(self, node, args, key, x=None):
        x = args[0] if x is None else x
        op = node.op_type
        if op == "Gelu":
            code = GELU_TANH if node.attr("approximate", "none") == "tanh" else GELU_ERF
            return self._map(code, x, key)
        if op == "Clip":
            lo = args[1] if len(args) > 1 and args[1] is not None else node.attr("min")
            hi = args[2] if len(args) > 2 and args[2] is not None else node.attr("max")
            lo = -np.inf if lo is None else float(np.asarray(lo).reshape(()))
            hi = np.inf if hi is None else float(np.asarray(hi).reshape(()))
            return self._map(CLIP, x, key, lo, hi)
        p0 = p1 = 0.0
        if op == "LeakyRelu":
            p0 = node.attr("alpha", 0.01)
        elif op == "HardSigmoid":
            p0, p1 = node.attr("alpha", 0.2), node.attr("beta", 0.5)
        elif op == "Elu":
            p0 = node.attr("alpha", 1.0)
        return self._map(MAP_OPS[op], x, key, p0, p1)

    def _fused(self, node, x, key):
        consts = node.attrs.get("consts", {})
        env = {node.inputs[0]: x}
        subs = node.attrs["nodes"]
        for i, sub in enumerate(subs):
            k = key if i == len(subs) - 1 else None
            sargs = [None if not n else env[n] if n in env else consts[n] for n in sub.inputs]
            if sub.op_type in BINARY_OPS:
                a = self._dev(sargs[0], (node.name, sub.inputs[0]))
                b = self._dev(sargs[1], (node.name, sub.inputs[1]))
                y = self._binary(sub.op_type, a, b, k)
            elif sub.op_type in MAP_OPS or sub.op_type in ("Gelu", "Clip"):
                y = self._unary(sub, sargs, k)
            else:
                raise UnsupportedGraph(f"'{sub.op_type}' inside FusedElementwise '{node.name}'")
            env[sub.outputs[0]] = y
        return env[node.outputs[0]]

    def _batchnorm(self, node, args, key):
        x = args[0]
        gamma, beta, mean, var = (np.asarray(v, dtype=np.float32) for v in args[1:5])
        a = gamma / np.sqrt(var + node.attr("epsilon", 1e-5))
        b = beta - a * mean
        shape = [1, -1] + [1] * (x.dim() - 2)
        ad = self._const((node.name, "a"), a.reshape(shape))
        bd = self._const((node.name, "b"), b.reshape(shape))
        y = self._binary("Mul", x, ad, None)
        return self._binary("Add", y, bd, key, out=y)

    def _layernorm(self, node, args, names, key):
        x = args[0]
        axis = float_ops._axis(node.attr("axis", -1), x.dim())
        D = int(np.prod(x.shape[axis:]))
        rows = x.numel() // D
        gamma = self._const(names[1], np.broadcast_to(np.asarray(args[1], np.float32),
                                                      x.shape[axis:]))
        beta = None
        if len(args) > 2 and args[2] is not None:
            beta = self._const(names[2], np.broadcast_to(np.asarray(args[2], np.float32),
                                                         x.shape[axis:]))
        y = self._empty(x.shape)
        self._call("qa_f32_layernorm_dev", x.data_ptr(), gamma.data_ptr(),
                   beta.data_ptr() if beta is not None else None, y.data_ptr(), rows, D,
                   float(node.attr("epsilon", 1e-5)), self._range_ptr(key))
        return y

    def _softmax(self, node, x, key):
        axis = softmax_axis(node, self.graph.opset, x.dim())
        if axis != x.dim() - 1:
            raise UnsupportedGraph("Softmax over an axis other than the last")
        cols = x.shape[-1]
        y = self._empty(x.shape)
        self._call("qa_f32_softmax_dev", x.data_ptr(), y.data_ptr(), x.numel() // cols, cols,
                   self._range_ptr(key))
        return y

    def _maxpool(self, node, x, key):
        N, C, H, W = x.shape
        (kh, kw), (sh, sw), (dh, dw), (pt, pl, pb, pr) = pool_geometry(node, tuple(x.shape))
        oh = (H + pt + pb - dh * (kh - 1) - 1) // sh + 1
        ow = (W + pl + pr - dw * (kw - 1) - 1) // sw + 1
        y = self._empty((N, C, oh, ow))
        self._call("qa_f32_maxpool_dev", x.data_ptr(), y.data_ptr(), N * C, H, W, kh, kw, sh,
                   sw, pt, pl, dh, dw, oh, ow, self._range_ptr(key))
        return y

    def _gap(self, x, key):
        N, C = x.shape[:2]
        hw = int(np.prod(x.shape[2:]))
        y = self._empty((N, C) + (1,) * (x.dim() - 2))
        self._call("qa_f32_plane_mean_dev", x.data_ptr(), y.data_ptr(), N * C, hw,
                   self._range_ptr(key))
        return y

    def _layout(self, node, args, keys):
        """Layout ops: the float op runs on a NumPy stand-in of the input's
        shape; each result is a view of it, whose offset and strides drive
        one strided copy on the device."""
        x = args[0]
        if not isinstance(x, torch.Tensor):
            raise UnsupportedGraph(f"{node.op_type} of a constant")
        proxy = np.empty(tuple(x.shape), dtype=np.float32)
        base = proxy.__array_interface__["data"][0]
        outs = float_ops.run_node(node, [proxy] + list(args[1:]), self.graph.opset)
        res = []
        for v, key in zip(outs, keys):
            if v.size and not np.may_share_memory(v, proxy):
                raise UnsupportedGraph(f"{node.op_type} result is not a view of its input")
            off = (v.__array_interface__["data"][0] - base) // 4
            y = self._empty(v.shape)
            if v.size:
                self._copy(x, y, v.shape, [s // 4 for s in v.strides], _dense_strides(v.shape),
                           x_off=off, key=key)
            res.append(y)
        return res

    def _concat(self, node, args, names, key):
        parts = [self._dev(a, n) for a, n in zip(args, names)]
        axis = float_ops._axis(node.attr("axis"), parts[0].dim())
        shape = list(parts[0].shape)
        shape[axis] = sum(p.shape[axis] for p in parts)
        y = self._empty(shape)
        ys = _dense_strides(shape)
        at = 0
        for p in parts:
            if p.numel():
                self._copy(p, y, p.shape, _dense_strides(p.shape), ys, y_off=at * ys[axis],
                           key=key)
            at += p.shape[axis]
        return y

    def _pad(self, node, args, key):
        x = args[0]
        pads = float_ops._attr_or_input(node, args, 1, "pads")
        pads = [int(p) for p in np.asarray(pads).reshape(-1)]
        n = x.dim()
        if any(p < 0 for p in pads):
            raise UnsupportedGraph("Pad with negative pads")
        if len(args) > 2 and args[2] is not None:
            value = float(np.asarray(args[2]).reshape(()))
        else:
            value = float(node.attr("value", 0))
        if (node.attr("mode", "constant") or "constant") not in ("constant", b"constant"):
            raise UnsupportedGraph("Pad mode other than constant")
        shape = [x.shape[i] + pads[i] + pads[i + n] for i in range(n)]
        y = self._empty(shape)
        ys = _dense_strides(shape)
        if any(pads):
            self._call("qa_f32_fill_dev", y.data_ptr(), y.numel(), value, self._range_ptr(key))
        off = sum(pads[i] * ys[i] for i in range(n))
        if x.numel():
            self._copy(x, y, x.shape, _dense_strides(x.shape), ys, y_off=off, key=key)
        return y

    def _expand(self, args, key):
        x = args[0] if isinstance(args[0], torch.Tensor) else self._dev(args[0])
        target = tuple(int(v) for v in np.asarray(args[1]).reshape(-1))
        shape = tuple(np.broadcast_shapes(tuple(x.shape), target))
        y = self._empty(shape)
        if y.numel():
            self._copy(x, y, shape, _broadcast_strides(x.shape, shape), _dense_strides(shape),
                       key=key)
        return y

    def _gather(self, node, args, key):
        x, idx = args[0], np.asarray(args[1]).astype(np.int64)
        if not isinstance(x, torch.Tensor) or isinstance(args[1], torch.Tensor):
            raise UnsupportedGraph("Gather needs a computed input and constant indices")
        axis = float_ops._axis(node.attr("axis", 0), x.dim())
        dim = x.shape[axis]
        flat = [int(i) + dim if i < 0 else int(i) for i in idx.reshape(-1)]
        xs = _dense_strides(x.shape)
        inner = list(x.shape[:axis]) + list(x.shape[axis + 1:])
        inner_strides = xs[:axis] + xs[axis + 1:]
        out_shape = list(x.shape[:axis]) + list(idx.shape) + list(x.shape[axis + 1:])
        y = self._empty(out_shape)
        # one copy per index: y[..., j, ...] = x[..., flat[j], ...]
        ys_full = _dense_strides([*x.shape[:axis], len(flat), *x.shape[axis + 1:]])
        ys = ys_full[:axis] + ys_full[axis + 1:]
        for j, i in enumerate(flat):
            self._copy(x, y, inner, inner_strides, ys, x_off=i * xs[axis],
                       y_off=j * ys_full[axis], key=key)
        return y

    # -------------------------------------------------------------- ranges --
    def packed(self):
        """The range table as float32 pairs (lo, -hi) on the device: the form
        one MIN all-reduce combines across ranks."""
        out = torch.empty((len(self.keys), 2), dtype=torch.float32, device=self.device)
        self._call("qa_f32_range_decode_dev", self.table.data_ptr(), out.data_ptr(),
                   len(self.keys))
        return out

    def allreduce(self, group=None):
        """Combines the range tables of all ranks on the device (one NCCL
        all-reduce, MIN of lows and of negated highs); returns the combined
        packed table."""
        import torch.distributed as dist

        packed = self.packed()
        dist.all_reduce(packed, op=dist.ReduceOp.MIN, group=group)
        return packed

    def ranges(self, packed=None):
        """``{key: (lo, hi)}`` of every observed tensor (one device-to-host
        copy).  A tensor never observed is left out; a NaN raises."""
        host = (packed if packed is not None else self.packed()).cpu().numpy().astype(np.float64)
        out = {}
        for k, (lo, neg_hi) in zip(self.keys, host):
            if np.isnan(lo) or np.isnan(neg_hi):
                raise ValueError(f"calibration tensor {k} holds NaN")
            if lo == np.inf and neg_hi == np.inf:
                continue  # not observed
            out[k] = (float(lo), float(-neg_hi))
        return out


def calibrate_on_device(container, batches, reduce_group=None, device=None, lib=None):
    """Observes ``batches`` on the GPU, merges the ranges the container
    already holds, combines across ``reduce_group``'s ranks on the device
    when given, sets them and finalizes (quant_container.py:75-112)."""
    batches = [batches] if isinstance(batches, (np.ndarray, dict)) else list(batches)
    if not batches:
        raise ValueError("no calibration data provided")
    cal = DeviceCalibrator(container, device, lib)
    for b in batches:
        cal.observe(b)
    packed = cal.allreduce(reduce_group) if reduce_group is not None else None
    ranges = cal.ranges(packed)
    for k, (lo, hi) in container.get_ranges().items():
        if k in ranges:
            ranges[k] = (min(lo, ranges[k][0]), max(hi, ranges[k][1]))
        else:
            ranges[k] = (lo, hi)
    container.set_ranges(ranges)
    container.finalize()
    return cal
