"""Device-resident, fused execution of a prepared QuantContainer.

The reference executes one layer at a time on host int32 arrays
(quant_container.py:135-193).  ResidentNet runs the same integer arithmetic
with every activation resident in HBM as int8 / uint8 NHWC bytes and with
the layer chain fused into few kernels:

* Conv / Gemm + requantize + activation LUT + residual Add + rescaled copy
  into a Concat slice -> one tensor-core launch (``qa_conv_fused_dev``);
* Split and Flatten -> zero-copy channel / shape views;
* Concat -> producers write straight into the concatenated buffer;
* GlobalAveragePool -> one reduction kernel; Softmax -> one float64
  fallback kernel that also emits the graph output's dequantized float32;
* graph-input quantization -> one kernel writing NHWC bytes.

All parameters come from the container's prepared layers (``w_centered``,
``bias_int``, ``q_mult``, ``shift``, ``lut``, ...), so results are bit-exact
with the reference's integer pass.  The launch sequence is captured once in
a CUDA graph; :meth:`ResidentNet.run` is the public host-to-host call
(pinned host input -> device -> output back to the host).
"""

import ctypes
from dataclasses import dataclass, field

import numpy as np
import torch

from quantanything_b200 import native
from quantanything_b200.layers import (
    ActivationQuantize,
    AddQuantize,
    BatchNormalizationQuantize,
    ConcatQuantize,
    ConvQuantize,
    GemmQuantize,
    GlobalAveragePoolQuantize,
    MulQuantize,
    ShapingQuantize,
)

_I64 = ctypes.c_int64
_P = ctypes.c_void_p


class FusedConvDesc(ctypes.Structure):
    """ctypes mirror of ``qa_fused_conv_desc`` (include/qa_kernels.h)."""

    _fields_ = [
        ("x", _P), ("x_pix_stride", _I64), ("x_signed", _I64), ("x_zp", _I64),
        ("N", _I64), ("H", _I64), ("W", _I64), ("C", _I64),
        ("KH", _I64), ("KW", _I64), ("SH", _I64), ("SW", _I64), ("PH", _I64), ("PW", _I64),
        ("DH", _I64), ("DW", _I64), ("OH", _I64), ("OW", _I64),
        ("Cout", _I64), ("groups", _I64),
        ("w", _P), ("w_rows", _I64), ("w_kp", _I64),
        ("bias", _P), ("mult", _P), ("shift", _P),
        ("zp", _I64), ("qmin", _I64), ("qmax", _I64), ("fast", _I64),
        ("lut", _P), ("lut_offset", _I64), ("lut_len", _I64),
        ("res", _P), ("res_pix_stride", _I64), ("res_signed", _I64),
        ("za", _I64), ("ma", _I64), ("sa", _I64), ("zb", _I64), ("mb", _I64), ("sb", _I64),
        ("sign", _I64), ("add_zo", _I64), ("add_qmin", _I64), ("add_qmax", _I64),
        ("out", _P), ("out_pix_stride", _I64),
        ("out2", _P), ("out2_pix_stride", _I64),
        ("r_identity", _I64), ("r_zp_in", _I64), ("r_m", _I64), ("r_s", _I64),
        ("r_zp_out", _I64), ("r_qmin", _I64), ("r_qmax", _I64),
        ("block_n", _I64),
        ("pad_corr", _P), ("pad_row_class", _P), ("pad_col_class", _P),
        ("pad_col_classes", _I64), ("pad_classes", _I64),
        ("gap_sum", _P), ("gap_cnt", _P), ("gap_out", _P), ("gap_out_stride", _I64),
        ("gap_zp_in", _I64), ("gap_mult", _I64), ("gap_shift", _I64), ("gap_zp_out", _I64),
        ("gap_qmin", _I64), ("gap_qmax", _I64),
    ]


_DEV_SIGNATURES = {
    "qa_conv_fused_dev": (ctypes.c_int, [ctypes.POINTER(FusedConvDesc), _P]),
    "qa_quantize_to_patch_rows_dev": (ctypes.c_int, [_P, _P] + [_I64] * 5 + [ctypes.c_double]
                                      + [_I64] * 3 + [_P]),
    "qa_quantize_to_nhwc_dev": (ctypes.c_int, [_P, _P] + [_I64] * 5 + [ctypes.c_double]
                                + [_I64] * 3 + [_P]),
    "qa_gap_dev": (ctypes.c_int, [_P] + [_I64] * 11 + [_P, _I64, _P]),
    "qa_softmax_dev": (ctypes.c_int, [_P, _I64, _I64, _I64, _I64, ctypes.c_double, _I64,
                                      ctypes.c_double, _I64, _I64, _I64, _P, _P,
                                      ctypes.c_double, _I64, _P]),
    "qa_lut_bytes_dev": (ctypes.c_int, [_P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _P, _I64,
                                        _P]),
    "qa_add_bytes_dev": (ctypes.c_int, [_P, _I64, _I64, _P, _I64, _I64, _P] + [_I64] * 13
                         + [_P]),
    "qa_rescale_bytes_dev": (ctypes.c_int, [_P, _I64, _I64, _P] + [_I64] * 10 + [_P]),
    "qa_mul_bytes_dev": (ctypes.c_int, [_P, _I64, _I64, _P, _I64, _I64, _P] + [_I64] * 10
                         + [_P]),
    "qa_bn_bytes_dev": (ctypes.c_int, [_P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _P, _P, _P,
                                       _I64, _I64, _I64, _P]),
    "qa_maxpool_bytes_dev": (ctypes.c_int, [_P, _I64, _I64, _P] + [_I64] * 16 + [_P]),
    "qa_bytes_to_i32_dev": (ctypes.c_int, [_P, _I64, _I64, _P, _I64, _I64, _I64, _P]),
    "qa_device_status_dev": (ctypes.c_int, [_P]),
    "qa_wait_probe_dev": (ctypes.c_int, [_I64, ctypes.c_int, _P]),
    "qa_window_copy_bytes_dev": (ctypes.c_int, [_P, _P] + [_I64] * 5 + [_P] * 4 + [_I64, _P]),
    "qa_matmul_act_bytes_dev": (ctypes.c_int, [_P, ctypes.c_int32, _I64, _I64, _I64, _I64,
                                               ctypes.c_double, _P, ctypes.c_int32, _I64, _I64,
                                               _I64, _I64, ctypes.c_double, _P, _I64, _I64,
                                               _I64, _I64, _I64, ctypes.c_double, _I64, _I64,
                                               _I64, _P]),
    "qa_requantize_i32_dev": (ctypes.c_int, [_P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _I64,
                                             _I64, _I64, _P]),
    "qa_conv_input_fused_dev": (ctypes.c_int, [ctypes.POINTER(FusedConvDesc), _P, _I64,
                                               ctypes.c_double, _I64, _I64, _P]),
    "qa_vit_embed_dev": (ctypes.c_int, [_P, _I64, ctypes.c_int32, _P, _P, _P, _I64, _I64, _P,
                                        _I64, _I64, _I64, _I64, _P]),
    "qa_layernorm_bytes_dev": (ctypes.c_int, [_P, _I64, ctypes.c_int32, _I64, ctypes.c_double,
                                              _P, _P, ctypes.c_double, ctypes.c_double, _I64,
                                              _I64, _I64, _P, _I64, _I64, _I64, _P]),
    "qa_attention_bytes_dev": (ctypes.c_int, [_P, _I64, ctypes.c_int32, _I64, ctypes.c_double,
                                              _I64, _I64, _I64, _I64, _P, _P, _P,
                                              ctypes.c_int32, _P, _I64, _P]),
    "qa_gather_table_dev": (ctypes.c_int, [_P, _I64, ctypes.c_int32, _I64, _I64, _P, _P, _I64,
                                           _I64, _I64, _P]),
    "qa_dequantize_rows_dev": (ctypes.c_int, [_P, _I64, ctypes.c_int32, _I64, ctypes.c_double,
                                              _P, _P, _I64, _I64, _P]),
}


WINDOW_OPS = ("Pad", "Slice", "Transpose")


def device_api(lib):
    """Declares the device-pointer entry points on a loaded KernelLibrary."""
    raw = lib.raw
    if not getattr(raw, "_qa_dev_declared", False):
        for name, (res, args) in _DEV_SIGNATURES.items():
            fn = getattr(raw, name)
            fn.restype, fn.argtypes = res, args
        raw._qa_dev_declared = True
    return raw


def _check(lib, rc, what):
    if rc != 0:
        msg = lib.raw.qa_last_error().decode(errors="replace")
        lib.raw.qa_clear_error()
        raise native.KernelLibraryError(f"{what}: {msg}")


def choose_block_n(cout, m_rows, taps_c, sm_count):
    """Column tile of the fused kernel: the output channels rounded up to a
    tile width (64 at most when the input is gathered 4 channels at a time);
    small-M layers take narrower tiles while the narrower tiling still fits
    one wave of the SMs (each CTA then gathers the same rows; L2 serves the
    repeats).  Halving into a second, partial wave costs more than it gains:
    measured on B200, the cfg0 Linear runs 12.3 us at 64 columns (96 tiles)
    against 13.9 us at 32 (192 tiles), and YOLOv8n-cls's 14x14 / 7x7 layers
    gain 1-3 us each."""
    bn = 16 if cout <= 16 else 32 if cout <= 32 else 64 if cout <= 64 else (
        128 if cout <= 128 else 256)
    if taps_c % 16 != 0:
        bn = min(bn, 64)
    m_tiles = -(-m_rows // 128)
    while bn > 32 and m_tiles * -(-cout // (bn // 2)) <= sm_count:
        bn //= 2
    return bn


def pad_corrections(wt, x_zp, H, W, KH, KW, SH, SW, PH, PW, DH, DW, OH, OW, max_classes=9):
    """Border correction tables of a padded conv whose input zero point is
    not 0 (the TMA gather reads out-of-image taps as 0 where the reference
    pads with the zero point): returns (corr [classes, Cout] int32, row class
    [OH] int32, column class [OW] int32, column classes) or None when no
    correction is needed or there are more than ``max_classes`` classes.
    ``wt`` holds the packed weights as [Cout, KH, KW, C] integers."""
    if x_zp == 0:
        return None
    rows = [tuple(ky for ky in range(KH) if not 0 <= oy * SH - PH + ky * DH < H)
            for oy in range(OH)]
    cols = [tuple(kx for kx in range(KW) if not 0 <= ox * SW - PW + kx * DW < W)
            for ox in range(OW)]
    rpat = sorted(set(rows), key=lambda t: (len(t), t))
    cpat = sorted(set(cols), key=lambda t: (len(t), t))
    if rpat == [()] and cpat == [()]:
        return None
    if len(rpat) * len(cpat) > max_classes or rpat[0] != () or cpat[0] != ():
        return None
    tapsum = np.asarray(wt, np.int64).sum(axis=3)  # [Cout, KH, KW]
    corr = np.zeros((len(rpat) * len(cpat), tapsum.shape[0]), np.int64)
    for i, rp in enumerate(rpat):
        for j, cp in enumerate(cpat):
            mask = np.zeros((KH, KW), bool)
            mask[list(rp), :] = True
            mask[:, list(cp)] = True
            corr[i * len(cpat) + j] = x_zp * tapsum[:, mask].sum(axis=1)
    if np.abs(corr).max() >= 1 << 30:
        return None
    row_class = np.array([rpat.index(t) for t in rows], np.int32)
    col_class = np.array([cpat.index(t) for t in cols], np.int32)
    return corr.astype(np.int32), row_class, col_class, len(cpat)


def window_geometry(node, graph, in_shape):
    """Pad / Slice / Transpose of a 4-D NCHW tensor as a window copy:
    (output shape, source axis, start, step) per output axis, following the
    reference's float ops (float_ops.py Pad: pads [begin..., end...] filled
    with the zero point; Slice: NumPy slicing of starts / ends / axes /
    steps, values beyond 2^62 meaning open ends; Transpose: perm, default
    reversed).  The batch axis must stay whole and in place."""
    from quantanything_b200.float_ops import _attr_or_input

    s = tuple(int(v) for v in in_shape)
    consts = [np.asarray(graph.initializers[i]) if i and graph.is_constant(i) else None
              for i in node.inputs]
    src, start, step, out = [0, 1, 2, 3], [0, 0, 0, 0], [1, 1, 1, 1], list(s)
    op = node.op_type
    if op == "Pad":
        pads = [int(v) for v in np.asarray(_attr_or_input(node, consts, 1, "pads")).reshape(-1)]
        if len(pads) != 8:
            raise UnsupportedGraph(f"{node.name}: Pad of a 4-D tensor expected")
        for a in range(4):
            start[a] = -pads[a]
            out[a] = s[a] + pads[a] + pads[a + 4]
    elif op == "Slice":
        starts = [int(v) for v in np.asarray(_attr_or_input(node, consts, 1, "starts")).reshape(-1)]
        ends = [int(v) for v in np.asarray(_attr_or_input(node, consts, 2, "ends")).reshape(-1)]
        axes = [int(v) for v in np.asarray(_attr_or_input(node, consts, 3, "axes",
                                                          list(range(len(starts))))).reshape(-1)]
        steps = [int(v) for v in np.asarray(_attr_or_input(node, consts, 4, "steps",
                                                           [1] * len(starts))).reshape(-1)]
        for st_, en, ax, sp in zip(starts, ends, axes, steps):
            a = ax % 4
            r = range(*slice(None if st_ >= 2**62 else st_, None if abs(en) >= 2**62 else en,
                             sp).indices(s[a]))
            start[a], step[a], out[a] = r.start, r.step, len(r)
    elif op == "Transpose":
        perm = [int(v) for v in (node.attr("perm") or [3, 2, 1, 0])]
        if sorted(perm) != [0, 1, 2, 3]:
            raise UnsupportedGraph(f"{node.name}: Transpose of a 4-D tensor expected")
        src = perm
        out = [s[a] for a in perm]
    else:
        raise AssertionError(op)
    if src[0] != 0 or start[0] != 0 or step[0] != 1 or out[0] != s[0] or min(out) <= 0:
        raise UnsupportedGraph(f"{node.name}: {op} must keep the batch axis and a non-empty "
                               "result")
    return tuple(out), src, start, step


def _round_up(v, m):
    return (v + m - 1) // m * m


@dataclass
class View:
    """An NHWC byte tensor (or a channel slice of one) resident on the GPU."""

    buf: torch.Tensor
    offset: int
    pix_stride: int
    N: int
    H: int
    W: int
    C: int
    signed: bool
    qp: object = None
    plane: int = 0  # 16-bit tensors: bytes from the low byte plane to the high one

    @property
    def ptr(self):
        return self.buf.data_ptr() + self.offset

    def channel_slice(self, c0, c):
        return View(self.buf, self.offset + c0, self.pix_stride, self.N, self.H, self.W, c,
                    self.signed, self.qp, self.plane)


@dataclass
class _ConvStep:
    layer: object
    desc: FusedConvDesc
    keep: list = field(default_factory=list)
    gap: tuple = None  # (layer, x, y, area) of a GlobalAveragePool fused into the epilogue


class UnsupportedGraph(NotImplementedError):
    """The graph has a layer the resident executor does not cover."""


class ResidentNet:
    """Fused device-resident integer inference of a prepared container."""

    _max_block_n = 256  # widest column tile of the contraction kernel

    def __init__(self, container, batch, device=None, fuse_input=True, fuse_gap=True):
        if not container.calibrated:
            raise ValueError("container is not calibrated")
        self.c = container
        self.graph = container.graph
        self.batch = int(batch)
        self.device = torch.device(device or "cuda")
        self.lib = container.lib
        device_api(self.lib)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.lib.set_device(self.device.index)
        self.sm_count = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.bits, self.signed = container.layers[0].num_bits, container.layers[0].signed
        self._check_bits()
        self.fuse_input = fuse_input
        self.fuse_gap = fuse_gap
        self._in_patch = 0  # > 0: the input quantizer writes patch rows (patch embedding)
        self._keep = []
        self.steps = []
        self.launch_count = 0
        self._graph = None
        self._plan()

    # ------------------------------------------------------------- helpers --
    def _check_bits(self):
        if self.bits > 8:
            raise UnsupportedGraph("the resident executor runs 8-bit graphs")

    def _operand_bits(self):
        """Width of the contraction operands (packed weights, activations)."""
        return self.bits


    def _weight_bits(self):
        """Signed width the packed centred weights must fit."""
        return self._operand_bits()
    def _alloc(self, nbytes):
        t = torch.empty(int(nbytes) + 64, dtype=torch.uint8, device=self.device)
        self._keep.append(t)
        return t

    def _dev(self, arr, dtype):
        t = torch.from_numpy(np.ascontiguousarray(arr, dtype=dtype)).to(self.device)
        self._keep.append(t)
        return t

    def _new_view(self, N, H, W, C, qp, pix_stride=None):
        stride = pix_stride or (C if C % 16 == 0 else _round_up(C, 16))
        return View(self._alloc(N * H * W * stride), 0, stride, N, H, W, C, self.signed, qp)

    # ---------------------------------------------------------------- plan --
    def _plan(self):
        g, c = self.graph, self.c
        layers = {l.name: l for l in c.layers}
        consumers = {}
        for node in g.nodes:
            for i in node.inputs:
                if i:
                    consumers.setdefault(i, []).append(node)
        self._consumers = consumers
        if len(g.inputs) != 1 or len(g.outputs) != 1:
            raise UnsupportedGraph("single-input single-output graphs only")
        in_name = g.inputs[0].name
        in_shape = g.inputs[0].shape
        self.in_shape = (self.batch, int(in_shape[1]), int(in_shape[2]), int(in_shape[3]))
        qp_in = c.qparams[in_name]
        Cin = self.in_shape[1]
        stride_in = Cin if Cin % 16 == 0 else _round_up(Cin, 4)
        views = {in_name: self._new_view(self.batch, self.in_shape[2], self.in_shape[3], Cin,
                                         qp_in, pix_stride=stride_in)}
        self.x_dev = torch.empty(self.in_shape, dtype=torch.float32, device=self.device)
        self.steps.append(("quantize", in_name))
        self._in_view = views[in_name]

        fused_away = set()   # layer names executed inside another layer's kernel
        concat_slot = {}     # tensor name -> (concat layer, input index)
        # Concat buffers are planned when the concat's first input is produced;
        # pre-compute every concat's output view up front (shapes from inputs).
        self._shapes = self._infer_shapes()
        for node in g.nodes:
            layer = layers[node.name]
            if isinstance(layer, ConcatQuantize):
                if node.attr("axis") not in (1, -3):
                    raise UnsupportedGraph("Concat must be along channels")
                N, C, H, W = self._shapes[node.outputs[0]]
                views[node.outputs[0]] = self._new_view(N, H, W, C, layer.out_qp[0])
                for idx, name in enumerate(node.inputs):
                    concat_slot.setdefault(name, []).append((layer, idx))
        self._concat_slot = concat_slot
        self._views = views
        self._concat_done = {}
        self._producer_step = {}

        for node in g.nodes:
            layer = layers[node.name]
            if node.name in fused_away:
                continue
            if isinstance(layer, (ConvQuantize, GemmQuantize)):
                self._plan_contraction(layer, layers, fused_away)
            elif isinstance(layer, ShapingQuantize) and node.op_type == "Split":
                self._plan_split(layer)
            elif isinstance(layer, ShapingQuantize) and node.op_type in ("Flatten", "Reshape",
                                                                         "Squeeze"):
                self._plan_flatten(layer)
            elif isinstance(layer, ConcatQuantize):
                self._plan_concat(layer)
            elif isinstance(layer, GlobalAveragePoolQuantize):
                self._plan_gap(layer)
            elif isinstance(layer, ShapingQuantize) and node.op_type == "MaxPool":
                self._plan_maxpool(layer)
            elif isinstance(layer, ShapingQuantize) and node.op_type in WINDOW_OPS:
                self._plan_window(layer)
            elif isinstance(layer, ActivationQuantize):
                self._plan_lut(layer)
            elif isinstance(layer, AddQuantize):
                self._plan_add(layer)
            elif isinstance(layer, MulQuantize):
                self._plan_mul(layer)
            elif isinstance(layer, BatchNormalizationQuantize):
                self._plan_bn(layer)
            elif node.op_type == "Softmax" and node.outputs[0] in g.outputs:
                self._plan_softmax(layer)
            else:
                raise UnsupportedGraph(f"{node.op_type} ({node.name}) has no resident kernel")
        out = g.outputs[0]
        if out not in self._outputs_f32:
            raise UnsupportedGraph("the graph output must be produced by the Softmax fallback")
        self._fuse_input_layer(in_name)

    def _fuse_input_layer(self, in_name):
        """Graph input -> first conv as one kernel (qa_conv_input_fused_dev:
        float patches by TMA, quantize in shared memory, tcgen05 MMA, fused
        epilogue), when ``fuse_input`` is set and the conv is the input's only
        reader with at most 4 input channels, at most 16 taps and no residual
        or concat copy, and its input tile fits the kernel's limits (the
        same checks the entry point makes)."""
        if (not self.fuse_input or len(self.steps) < 2 or self.steps[0][0] != "quantize"
                or self.steps[1][0] != "conv"):
            return
        step = self.steps[1][1]
        d = step.desc
        readers = self._consumers.get(in_name, [])
        if (len(readers) != 1 or readers[0] is not step.layer.node or d.groups != 1 or d.C != 4
                or self.in_shape[1] > 4 or d.KH * d.KW > 16 or self.in_shape[3] % 4
                or not d.x_signed or d.Cout > 64 or d.res or d.out2 or not d.out
                or d.qmin < -128 or d.qmax > 255):
            return
        patch_h = 15 * d.SH + (d.KH - 1) * d.DH + 1
        patch_w = 27 * d.SW + (d.KW - 1) * d.DW + 1
        box_w = _round_up(patch_w + (-d.PW) % 4, 4)
        cout_p = _round_up(d.Cout, 16)
        stage = _round_up(self.in_shape[1] * patch_h * box_w * 4, 1024)
        smem = (1024 + 2 * stage + 4 * 128 * 64 + cout_p * 64 + cout_p * 40 + 384 * 4 + 64
                + patch_h * patch_w * 4 + 48)
        if box_w > 256 or patch_h > 256 or patch_h * patch_w >= 65536 or smem > 110 * 1024:
            return
        self.steps[0:2] = [("conv_input", step)]

    # --------------------------------------------------------- shape pass --
    def _infer_shapes(self):
        g, layers = self.graph, {l.name: l for l in self.c.layers}
        shapes = {g.inputs[0].name: self.in_shape}
        for node in g.nodes:
            layer = layers[node.name]
            ins = [shapes.get(i) for i in node.inputs if i]
            s = ins[0]
            if isinstance(layer, ConvQuantize):
                strides, pads, dil, groups = layer.geometry(s)
                g_ = native.conv_geometry(s, layer.w_q.shape, strides, pads, dil, groups)
                shapes[node.outputs[0]] = (s[0], layer.w_q.shape[0], g_[13], g_[14])
            elif isinstance(layer, GemmQuantize):
                shapes[node.outputs[0]] = (s[0], layer.w_q.shape[1], 1, 1)
            elif node.op_type == "Split":
                sizes = list(np.asarray(g.initializers[node.inputs[1]]).reshape(-1)) if len(
                    node.inputs) > 1 and node.inputs[1] else [s[1] // len(node.outputs)] * len(
                    node.outputs)
                for o, sz in zip(node.outputs, sizes):
                    shapes[o] = (s[0], int(sz), s[2], s[3])
            elif node.op_type == "Concat":
                shapes[node.outputs[0]] = (s[0], sum(x[1] for x in ins), s[2], s[3])
            elif node.op_type == "GlobalAveragePool":
                shapes[node.outputs[0]] = (s[0], s[1], 1, 1)
            elif node.op_type in ("Flatten", "Reshape", "Squeeze"):
                shapes[node.outputs[0]] = (s[0], s[1] * s[2] * s[3], 1, 1)
            elif node.op_type in WINDOW_OPS:
                shapes[node.outputs[0]] = window_geometry(node, g, s)[0]
            elif node.op_type == "MaxPool":
                from quantanything_b200.float_ops import pool_geometry

                k, st, dl, pd = pool_geometry(node, s)
                oh = (s[2] + pd[0] + pd[2] - dl[0] * (k[0] - 1) - 1) // st[0] + 1
                ow = (s[3] + pd[1] + pd[3] - dl[1] * (k[1] - 1) - 1) // st[1] + 1
                shapes[node.outputs[0]] = (s[0], s[1], oh, ow)
            else:
                shapes[node.outputs[0]] = s
        return shapes

    # ------------------------------------------------------- destinations --
    def _only_consumer(self, tensor):
        cons = self._consumers.get(tensor, [])
        return cons[0] if len(cons) == 1 and tensor not in self.graph.outputs else None

    def _destination(self, tensor, qp, N, H, W, C):
        """(primary view or None, concat copy spec or None) for a produced tensor.

        A tensor whose only consumer is a Concat on the same grid is written
        straight into the concat slice; one with other consumers gets its own
        buffer plus a (rescaled) copy into the slice."""
        slots = self._concat_slot.get(tensor, [])
        cons = self._consumers.get(tensor, [])
        copy = None
        if slots:
            concat, idx = slots[0]
            out_view = self._views[concat.node.outputs[0]]
            c0 = sum(self._shapes[n][1] for n in concat.node.inputs[:idx])
            slice_view = out_view.channel_slice(c0, C)
            if len(cons) == 1 and concat.same_grid(idx):
                self._concat_done[(concat.name, idx)] = True
                return slice_view, None
            copy = (concat, idx, slice_view)
        view = self._new_view(N, H, W, C, qp)
        return view, copy

    # ------------------------------------------------------ contractions --
    def _pack_weights(self, layer, x_view, taps_c, m_rows):
        if isinstance(layer, GemmQuantize):
            wc = np.ascontiguousarray(layer.w_centered.T).astype(np.int64)  # [N, K]
            cout, kh, kw, groups, cg = wc.shape[0], 1, 1, 1, wc.shape[1]
            w4 = wc.reshape(cout, cg, 1, 1)
        else:
            w4 = layer.w_centered.astype(np.int64)
            cout, cg, kh, kw = w4.shape
            groups = layer.node.attr("group", 1)
        bits = self._weight_bits()
        lim = 1 << (bits - 1)
        if w4.min() < -lim or w4.max() >= lim:
            raise UnsupportedGraph(f"{layer.name}: centred weights exceed int{bits}")
        ct = taps_c if groups == 1 else cg
        bn = min(choose_block_n(cout, m_rows, ct if groups == 1 else 16, self.sm_count),
                 self._max_block_n)
        rows = _round_up(cout, bn)
        k = kh * kw * ct
        kp = _round_up(k, 16)
        packed = np.zeros((rows, kp), np.int8 if bits == 8 else np.int16 if bits == 16
                          else np.int32)
        wt = np.zeros((cout, kh, kw, ct), np.int64)
        wt[:, :, :, :cg] = np.transpose(w4, (0, 2, 3, 1))
        packed[:cout, :k] = wt.reshape(cout, k)
        colsum = wt.reshape(cout, k).sum(axis=1)
        abssum = np.abs(wt.reshape(cout, k)).sum(axis=1)
        return packed, rows, kp, bn, groups, ct, colsum, abssum

    def _upload_weights(self, packed):
        return self._dev(packed, np.int8)

    def _plan_contraction(self, layer, layers, fused_away, patch=0):
        """``patch`` > 0: the input view holds the im2col rows of this
        patch x patch, stride-patch conv (written by the input quantizer), so
        the layer runs as a pointwise GEMM over those rows with the conv's own
        packed weights (K = patch * patch * 4)."""
        node = layer.node
        x_view = self._views[node.inputs[0]]
        N, _, H, W = self._shapes[node.inputs[0]]
        if patch:
            cin = int(layer.w_q.shape[1])
            strides, pads, dil, groups = layer.geometry((N, cin, H, W))
            g_ = native.conv_geometry((N, cin, H, W), layer.w_q.shape, strides, pads, dil, groups)
            m_rows = N * g_[13] * g_[14]
            packed, rows, kp, bn, groups, ct, colsum, abssum = self._pack_weights(layer, x_view,
                                                                                  4, m_rows)
            geo = dict(KH=1, KW=1, SH=1, SW=1, PH=0, PW=0, DH=1, DW=1, OH=g_[13], OW=g_[14])
            H, W, ct_desc = g_[13], g_[14], g_[5] * g_[6] * 4
            pads_bottom = (0, 0)
            # column tile of a 16-byte-aligned row matrix (the packing above
            # chose one for 4-byte taps)
            cout_ = int(layer.w_q.shape[0])
            bn = choose_block_n(cout_, m_rows, 16, self.sm_count)
            rows = _round_up(cout_, bn)
            if rows != packed.shape[0]:
                packed = np.concatenate(
                    [packed[:cout_], np.zeros((rows - cout_, packed.shape[1]), packed.dtype)])
        elif isinstance(layer, GemmQuantize):
            if (x_view.H, x_view.W) != (1, 1):
                raise UnsupportedGraph("Gemm input must be a flattened vector")
            geo = dict(KH=1, KW=1, SH=1, SW=1, PH=0, PW=0, DH=1, DW=1, OH=1, OW=1)
            pads_bottom = (0, 0)
        else:
            strides, pads, dil, groups = layer.geometry((N, x_view.C, H, W))
            g_ = native.conv_geometry((N, x_view.C, H, W), layer.w_q.shape, strides, pads, dil,
                                      groups)
            geo = dict(KH=g_[5], KW=g_[6], SH=g_[7], SW=g_[8], PH=g_[9], PW=g_[10], DH=g_[11],
                       DW=g_[12], OH=g_[13], OW=g_[14])
            pads_bottom = (pads[2], pads[3])
        if not patch:
            taps_c = x_view.C
            if taps_c % 16 != 0:
                taps_c = _round_up(taps_c, 4)
                if taps_c > x_view.pix_stride and x_view.offset + taps_c > x_view.pix_stride:
                    raise UnsupportedGraph(f"{layer.name}: input channels not 4-aligned")
            m_rows = N * geo["OH"] * geo["OW"]
            packed, rows, kp, bn, groups, ct, colsum, abssum = self._pack_weights(
                layer, x_view, taps_c, m_rows)
            ct_desc = ct
        cout = layer.w_q.shape[1] if isinstance(layer, GemmQuantize) else layer.w_q.shape[0]
        x_zp = layer.in_zp
        bias = (layer.bias_int.astype(np.int64) if layer.bias_int is not None
                else np.zeros(cout, np.int64)) - x_zp * colsum
        mult = np.broadcast_to(np.asarray(layer.q_mult, np.int64), (cout,)).copy()
        shift = np.broadcast_to(np.asarray(layer.shift, np.int64), (cout,)).copy()
        xmax = max(abs(layer.in_qmin), abs(layer.in_qmax))
        # (|x_zp| * abssum covers the border corrections of the TMA gather)
        bound = xmax * abssum + np.abs(bias) + abs(int(x_zp)) * abssum
        ts = 31 + shift
        # 64-bit requantize is exact when acc + bias and M0 fit int32 and the
        # rounded product cannot overflow (checked per channel, exact ints)
        fast = bool(np.all((ts >= 1) & (ts <= 62)) and all(
            int(b) < (1 << 31) and abs(int(m)) < (1 << 31) and abs(int(bi)) < (1 << 31)
            and int(b) * abs(int(m)) + (1 << (int(t) - 1)) < (1 << 62)
            for b, m, t, bi in zip(bound, mult, ts, bias)))
        d = FusedConvDesc()
        d.x, d.x_pix_stride, d.x_signed, d.x_zp = x_view.ptr, x_view.pix_stride, int(
            x_view.signed), int(x_zp)
        d.N, d.H, d.W, d.C = N, H, W, ct_desc
        for k_, v in geo.items():
            setattr(d, k_, int(v))
        d.Cout, d.groups = cout, groups
        wdev = self._upload_weights(packed)
        d.w, d.w_rows, d.w_kp = wdev.data_ptr(), rows, kp
        bdev, mdev, sdev = (self._dev(bias, np.int64), self._dev(mult, np.int64),
                            self._dev(shift, np.int64))
        d.bias, d.mult, d.shift = bdev.data_ptr(), mdev.data_ptr(), sdev.data_ptr()
        d.zp, d.qmin, d.qmax, d.fast = layer.out_zp, layer.out_qmin, layer.out_qmax, int(fast)
        d.block_n = bn if groups == 1 else 0
        if (groups == 1 and ct % 16 == 0 and x_zp != 0 and not patch
                and self._operand_bits() == 8):
            wt = packed[:cout, :geo["KH"] * geo["KW"] * ct].reshape(cout, geo["KH"], geo["KW"], ct)
            pc = pad_corrections(wt, int(x_zp), H, W, **geo)
            if pc is not None:
                corr, rcls, ccls, ncol = pc
                d.pad_corr = self._dev(corr, np.int32).data_ptr()
                d.pad_row_class = self._dev(rcls, np.int32).data_ptr()
                d.pad_col_class = self._dev(ccls, np.int32).data_ptr()
                d.pad_col_classes, d.pad_classes = ncol, corr.shape[0]
        produced = node.outputs[0]
        out_qp = layer.out_qp[0]
        # activation LUT fused when it is the only consumer
        act = self._only_consumer(produced)
        if act is not None and isinstance(layers[act.name], ActivationQuantize):
            a = layers[act.name]
            ldev = self._dev(a.lut, np.int32)
            d.lut, d.lut_offset, d.lut_len = ldev.data_ptr(), int(a.lut_offset), len(a.lut)
            fused_away.add(act.name)
            produced, out_qp = act.outputs[0], a.out_qp[0]
        # residual Add fused when it is the only consumer (of the LUT output, or
        # of the contraction itself)
        add = self._only_consumer(produced)
        if add is not None and isinstance(layers[add.name], AddQuantize):
            al = layers[add.name]
            other = [i for i in add.inputs if i != produced]
            if len(other) == 1 and other[0] in self._views and (
                    add.inputs[1] == produced or al._sign == 1):
                res = self._views[other[0]]
                (ma, sa), (mb, sb) = al._mult
                qa, qb = al.in_qp
                if add.inputs[1] == produced:  # out = res (a) + sign * ours (b)
                    d.za, d.ma, d.sa, d.zb, d.mb, d.sb = qa.zp, ma, sa, qb.zp, mb, sb
                else:  # ours is operand a, sign == +1: the sum commutes
                    d.za, d.ma, d.sa, d.zb, d.mb, d.sb = qb.zp, mb, sb, qa.zp, ma, sa
                d.res, d.res_pix_stride, d.res_signed = res.ptr, res.pix_stride, int(
                    res.signed)
                o = al.out_qp[0]
                d.sign, d.add_zo, d.add_qmin, d.add_qmax = al._sign, o.zp, o.qmin, o.qmax
                fused_away.add(add.name)
                produced, out_qp = add.outputs[0], o
        NO, HO, WO = (N, geo["OH"], geo["OW"])
        view, copy = self._destination(produced, out_qp, NO, HO, WO, cout)
        if view is not None and (self._consumers.get(produced) or produced in self.graph.outputs
                                 or copy is None):
            d.out, d.out_pix_stride = view.ptr, view.pix_stride
            self._views[produced] = view
        if copy is not None:
            concat, idx, sl = copy
            self._attach_copy(d, concat, idx, sl)
            cons = self._consumers.get(produced, [])
            if len(cons) == 1:  # the concat is the only reader: no primary store
                d.out = None
        step = _ConvStep(layer, d)
        self._producer_step[produced] = step
        self.steps.append(("conv", step))

    def _attach_copy(self, d, concat, idx, slice_view):
        (m, s) = concat._mult[idx]
        qp, o = concat.in_qp[idx], concat.out_qp[0]
        d.out2, d.out2_pix_stride = slice_view.ptr, slice_view.pix_stride
        d.r_identity = int(concat.same_grid(idx))
        d.r_zp_in, d.r_m, d.r_s, d.r_zp_out, d.r_qmin, d.r_qmax = qp.zp, m, s, o.zp, o.qmin, o.qmax
        self._concat_done[(concat.name, idx)] = True

    # --------------------------------------------------------- other ops --
    def _plan_split(self, layer):
        node = layer.node
        src = self._views[node.inputs[0]]
        c0 = 0
        for o in node.outputs:
            C = self._shapes[o][1]
            self._views[o] = src.channel_slice(c0, C)
            c0 += C
        # Split outputs that land, in order, in consecutive slots of one
        # Concat (the C2f pattern) are copied by the producer of the split
        # input as a single rescaled second output; otherwise _plan_concat
        # emits standalone copies.
        step = self._producer_step.get(node.inputs[0])
        if step is None or step.desc.out2:
            return
        slots = [self._concat_slot.get(o, []) for o in node.outputs]
        if any(len(sl) != 1 for sl in slots):
            return
        concat = slots[0][0][0]
        idxs = [sl[0][1] for sl in slots]
        if any(sl[0][0] is not concat for sl in slots) or idxs != list(
                range(idxs[0], idxs[0] + len(idxs))):
            return
        if any(concat._mult[i] != concat._mult[idxs[0]]
               or concat.same_grid(i) != concat.same_grid(idxs[0]) for i in idxs):
            return
        if c0 != src.C:
            return
        start = sum(self._shapes[n][1] for n in concat.node.inputs[:idxs[0]])
        out = self._views[concat.node.outputs[0]]
        self._attach_copy(step.desc, concat, idxs[0], out.channel_slice(start, c0))
        for i in idxs:
            self._concat_done[(concat.name, i)] = True

    def _plan_flatten(self, layer):
        node = layer.node
        src = self._views[node.inputs[0]]
        if (src.H, src.W) != (1, 1):
            if src.pix_stride != src.C:
                raise UnsupportedGraph("Flatten of a strided spatial tensor")
            raise UnsupportedGraph("Flatten of a spatial tensor (NCHW order) is not resident")
        self._views[node.outputs[0]] = src

    def _plan_concat(self, layer):
        node = layer.node
        out = self._views[node.outputs[0]]
        c0 = 0
        for idx, name in enumerate(node.inputs):
            C = self._shapes[name][1]
            if not self._concat_done.get((layer.name, idx)):
                self.steps.append(("rescale", (layer, idx, self._views[name],
                                               out.channel_slice(c0, C))))
            c0 += C

    def _plan_gap(self, layer):
        node = layer.node
        x = self._views[node.inputs[0]]
        N, C, H, W = self._shapes[node.inputs[0]]
        view, copy = self._destination(node.outputs[0], layer.out_qp[0], N, 1, 1, C)
        if copy is not None:
            raise UnsupportedGraph("GlobalAveragePool feeding a Concat")
        self._views[node.outputs[0]] = view
        if not self._fuse_gap(layer, x, view, H * W):
            self.steps.append(("gap", (layer, x, view, H * W)))

    def _fuse_gap(self, layer, x, view, hw):
        """GlobalAveragePool (quant_layers.py:563-590) folded into the epilogue
        of the pointwise contraction that produces its input (the head conv
        of YOLOv8n-cls): the epilogue sums each image's (v - zp_in) per
        channel and the warp that completes an (image, column tile)
        requantizes it, so the pooled tensor needs no separate launch and
        the layer output is not read again.  8-bit graphs only; the
        producer must be a pointwise conv with a 128 or 256 column tile
        whose only reader is this pool, and an image must cover at least 32
        pixels (a warp's rows then span at most two images)."""
        if not self.fuse_gap or self._operand_bits() != 8:
            return False
        src = layer.node.inputs[0]
        step = self._producer_step.get(src)
        if step is None or src in self.graph.outputs or len(self._consumers.get(src, [])) != 1:
            return False
        d = step.desc
        if (d.groups != 1 or d.KH != 1 or d.KW != 1 or d.SH != 1 or d.SW != 1 or d.PH or d.PW
                or d.C % 16 or d.x_pix_stride % 16 or d.out2 or d.gap_sum
                or d.block_n not in (128, 256) or hw < 32 or hw * 255 >= 2**31
                or not d.out or d.out != x.ptr or not (-128 <= layer.in_zp <= 255)):
            return False
        m, s = layer.multiplier(hw)
        n_tiles = -(-int(d.Cout) // int(d.block_n))
        sums = torch.zeros((x.N, int(d.Cout)), dtype=torch.int32, device=self.device)
        counts = torch.zeros((x.N, n_tiles), dtype=torch.int32, device=self.device)
        self._keep += [sums, counts]
        self._gap_scratch = getattr(self, "_gap_scratch", []) + [sums, counts]
        d.gap_sum, d.gap_cnt = sums.data_ptr(), counts.data_ptr()
        d.gap_out, d.gap_out_stride = view.ptr, view.pix_stride
        d.gap_zp_in, d.gap_mult, d.gap_shift = int(layer.in_zp), int(m), int(s)
        d.gap_zp_out, d.gap_qmin, d.gap_qmax = layer.out_zp, layer.out_qmin, layer.out_qmax
        step.gap = (layer, x, view, hw)
        return True

    def _plan_maxpool(self, layer):
        node = layer.node
        x = self._views[node.inputs[0]]
        N, C, OH, OW = self._shapes[node.outputs[0]]
        view, copy = self._destination(node.outputs[0], layer.out_qp[0], N, OH, OW, C)
        self._views[node.outputs[0]] = view
        self.steps.append(("maxpool", (layer, x, view)))
        if copy is not None:
            self.steps.append(("rescale", (copy[0], copy[1], view, copy[2])))

    def _plan_window(self, layer):
        """Pad / Slice / Transpose (quant_layers.py:593-650, scale preserving;
        Pad fills with the input zero point): a channel Slice of step 1 on
        16-byte boundaries is a view of its input, any other form one window
        copy (qa_window_copy_bytes_dev) into a new tensor."""
        node = layer.node
        x = self._views[node.inputs[0]]
        s = self._shapes[node.inputs[0]]
        out_shape, src, start, step = window_geometry(node, self.graph, s)
        N, C, H, W = out_shape
        channel_view = (node.op_type == "Slice" and src == [0, 1, 2, 3] and step[1] == 1
                        and (out_shape[2], out_shape[3]) == (s[2], s[3])
                        and start[1] % 16 == 0 and C % 16 == 0
                        and node.outputs[0] not in self._concat_slot)
        if channel_view:
            self._views[node.outputs[0]] = x.channel_slice(start[1], C)
            return
        view, copy = self._destination(node.outputs[0], layer.out_qp[0], N, H, W, C)
        self._views[node.outputs[0]] = view
        ps = x.pix_stride
        src_stride = [s[2] * s[3] * ps, 1, s[3] * ps, ps]  # NCHW axes of the NHWC source
        geom = np.array([start, step, [s[a] for a in src], [src_stride[a] for a in src]],
                        np.int64)
        self.steps.append(("window", (layer, x, view, geom, int(layer.in_zp))))
        if copy is not None:
            self.steps.append(("rescale", (copy[0], copy[1], view, copy[2])))

    def _plan_lut(self, layer):
        node = layer.node
        x = self._views[node.inputs[0]]
        N, C, H, W = self._shapes[node.outputs[0]]
        view, copy = self._destination(node.outputs[0], layer.out_qp[0], N, H, W, C)
        self._views[node.outputs[0]] = view
        self.steps.append(("lut", (layer, x, view, self._dev(layer.lut, np.int32))))
        if copy is not None:
            self.steps.append(("rescale", (copy[0], copy[1], view, copy[2])))

    def _plan_add(self, layer):
        node = layer.node
        a, b = (self._views[i] for i in node.inputs)
        N, C, H, W = self._shapes[node.outputs[0]]
        view, copy = self._destination(node.outputs[0], layer.out_qp[0], N, H, W, C)
        self._views[node.outputs[0]] = view
        self.steps.append(("add", (layer, a, b, view)))
        if copy is not None:
            self.steps.append(("rescale", (copy[0], copy[1], view, copy[2])))

    def _plan_mul(self, layer):
        node = layer.node
        a, b = (self._views[i] for i in node.inputs)
        N, C, H, W = self._shapes[node.outputs[0]]
        view, copy = self._destination(node.outputs[0], layer.out_qp[0], N, H, W, C)
        self._views[node.outputs[0]] = view
        self.steps.append(("mul", (layer, a, b, view)))
        if copy is not None:
            self.steps.append(("rescale", (copy[0], copy[1], view, copy[2])))

    def _plan_bn(self, layer):
        node = layer.node
        x = self._views[node.inputs[0]]
        N, C, H, W = self._shapes[node.outputs[0]]
        view, copy = self._destination(node.outputs[0], layer.out_qp[0], N, H, W, C)
        self._views[node.outputs[0]] = view
        params = [self._dev(np.broadcast_to(np.asarray(v, np.int64), (C,)).copy(), np.int64)
                  for v in (layer.q_mult, layer.shift, layer.q_B)]
        self.steps.append(("bn", (layer, x, view, params)))
        if copy is not None:
            self.steps.append(("rescale", (copy[0], copy[1], view, copy[2])))

    def _plan_softmax(self, layer):
        node = layer.node
        x = self._views[node.inputs[0]]
        N, C = self._shapes[node.inputs[0]][:2]
        self.out_f32 = torch.empty((N, C), dtype=torch.float32, device=self.device)
        self.out_q = torch.empty((N, C), dtype=torch.int32, device=self.device)
        self._outputs_f32 = {node.outputs[0]: self.out_f32}
        self.steps.append(("softmax", (layer, x)))

    _outputs_f32 = {}

    # --------------------------------------------------------------- costs --
    def step_costs(self):
        """Algorithmic (bytes moved, integer ops) of every step: each tensor
        counted once (activations as stored bytes, weights once per launch),
        ops = 2 * MACs of the contraction."""
        costs = []
        for kind, payload in self.steps:
            if kind == "quantize":
                N, C, H, W = self.in_shape
                v = self._in_view
                costs.append((f"quantize {N}x{C}x{H}x{W}", N * C * H * W * 4 +
                              N * H * W * (4 if self._in_patch else v.pix_stride), 0))
            elif kind in ("conv", "conv_input"):
                d = payload.desc
                M = d.N * d.OH * d.OW
                cg = d.C
                k = d.KH * d.KW * cg
                x_bytes = d.N * d.H * d.W * (cg * d.groups if d.groups > 1 else cg)
                if kind == "conv_input":  # float32 images, 3 channels read
                    x_bytes = d.N * d.H * d.W * self.in_shape[1] * 4
                stores = (1 if d.out else 0) + (1 if d.out2 else 0) + (1 if d.res else 0)
                nbytes = x_bytes + d.Cout * k + M * d.Cout * stores + d.Cout * 24
                ops = 2 * M * d.Cout * (d.KH * d.KW * cg)
                label = (f"{payload.layer.node.op_type.lower()} {d.KH}x{d.KW}/s{d.SH} "
                         f"{cg * d.groups}->{d.Cout} @{d.OH}x{d.OW}")
                if kind == "conv_input":
                    label = "quantize+" + label
                if getattr(payload, "gap", None) is not None:
                    label += "+gap"
                    nbytes += d.N * d.Cout  # the pooled bytes
                costs.append((label, nbytes, ops))
            elif kind == "gap":
                layer, x, y, area = payload
                costs.append((f"gap {x.C}@{x.H}x{x.W}", x.N * area * x.C + x.N * x.C, 0))
            elif kind == "softmax":
                layer, x = payload
                costs.append((f"softmax {x.N}x{x.C}", x.N * x.C * 9, 0))
            elif kind == "window":
                layer, x, y = payload[:3]
                costs.append((f"{layer.node.op_type.lower()} {y.C}@{y.H}x{y.W}",
                              2 * y.N * y.H * y.W * y.C, 0))
            else:
                src = payload[1] if kind != "rescale" else payload[2]
                rows = src.N * src.H * src.W
                costs.append((kind, rows * src.C * 2, 0))
        return costs

    def time_steps(self, reps=20):
        """Average device time (ms) of every step over ``reps`` eager runs,
        measured with CUDA events recorded between the launches on the
        launching stream."""
        stream = torch.cuda.current_stream(self.device)
        totals = np.zeros(len(self.steps))
        for _ in range(reps):
            events = [torch.cuda.Event(enable_timing=True) for _ in range(len(self.steps) + 1)]

            def mark(i, events=events):
                events[i + 1].record(stream)

            events[0].record(stream)
            self._launch_all(stream.cuda_stream, on_step=mark)
            stream.synchronize()
            totals += [events[i].elapsed_time(events[i + 1]) for i in range(len(self.steps))]
        return totals / reps

    def time_steps_graphed(self, reps=20, flush=None):
        """Device time (ms) of every step, each captured alone in a CUDA graph
        (so host-side launch work is not timed) and replayed ``reps`` times,
        with CUDA events around each replay on the replaying stream;
        ``flush`` (a device tensor, zeroed before every replay outside the
        events) takes the step's inputs out of L2.  Returns the mean per
        step."""
        torch.cuda.synchronize(self.device)
        self.forward_device()  # eager warm-up: one-time host preparation
        torch.cuda.synchronize(self.device)
        saved = self.steps
        totals = np.zeros(len(saved))
        s = torch.cuda.Stream(self.device)
        try:
            for i, step in enumerate(saved):
                self.steps = [step]
                g = torch.cuda.CUDAGraph()
                with torch.cuda.stream(s):
                    with torch.cuda.graph(g, stream=s):
                        self._launch_all(s.cuda_stream)
                torch.cuda.synchronize(self.device)
                for _ in range(reps):
                    with torch.cuda.stream(s):
                        if flush is not None:
                            flush.zero_()
                        e0 = torch.cuda.Event(enable_timing=True)
                        e1 = torch.cuda.Event(enable_timing=True)
                        e0.record(s)
                        g.replay()
                        e1.record(s)
                    e1.synchronize()
                    totals[i] += e0.elapsed_time(e1)
                del g
        finally:
            self.steps = saved
            self.launch_count = len(saved)
        return totals / reps

    def time_steps_in_graph(self, flush, repeat=10, reps=5):
        """Device time (ms) of every step, from one CUDA graph holding
        ``repeat`` rounds of (zero ``flush``, launch the step) against one
        holding the ``repeat`` flushes alone: the difference of their replay
        times (median of ``reps``) over ``repeat``.  Each launch starts with
        its inputs out of L2, as in :meth:`time_steps_graphed`, but the graph
        launch and the granularity of the event timestamps (single-replay
        figures fell on a 2.048 µs grid on B200) are spread over ``repeat``
        launches; what remains is the launch's own time after the flush
        kernel it depends on."""
        torch.cuda.synchronize(self.device)
        self.forward_device()  # eager warm-up: one-time host preparation
        torch.cuda.synchronize(self.device)
        saved = self.steps
        out = np.zeros(len(saved))
        s = torch.cuda.Stream(self.device)

        def replay_ms(g):
            with torch.cuda.stream(s):
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(s)
                g.replay()
                e1.record(s)
            e1.synchronize()
            return e0.elapsed_time(e1)

        try:
            g0 = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s):
                with torch.cuda.graph(g0, stream=s):
                    for _ in range(repeat):
                        flush.zero_()
            for i, step in enumerate(saved):
                self.steps = [step]
                g1 = torch.cuda.CUDAGraph()
                with torch.cuda.stream(s):
                    with torch.cuda.graph(g1, stream=s):
                        for _ in range(repeat):
                            flush.zero_()
                            self._launch_all(s.cuda_stream)
                torch.cuda.synchronize(self.device)
                t1, t0 = [], []
                for _ in range(reps):
                    t1.append(replay_ms(g1))
                    t0.append(replay_ms(g0))
                out[i] = max(float(np.median(t1) - np.median(t0)), 0.0) / repeat
                del g1
            del g0
        finally:
            self.steps = saved
            self.launch_count = len(saved)
        return out

    # ------------------------------------------------------------- launch --
    def _launch_all(self, stream, on_step=None):
        raw = self.lib.raw
        raw.qa_set_device(self.device.index)  # launches go to this executor's GPU
        st = ctypes.c_void_p(stream)
        n = 0
        for kind, payload in self.steps:
            if kind == "quantize":
                v, qp = self._in_view, self.c.qparams[payload]
                N, C, H, W = self.in_shape
                if self._in_patch:
                    rc = raw.qa_quantize_to_patch_rows_dev(
                        self.x_dev.data_ptr(), v.ptr, N, C, H, W, self._in_patch,
                        float(qp.scale), qp.zp, qp.qmin, qp.qmax, st)
                else:
                    rc = raw.qa_quantize_to_nhwc_dev(self.x_dev.data_ptr(), v.ptr, N, C, H, W,
                                                     v.pix_stride, float(qp.scale), qp.zp,
                                                     qp.qmin, qp.qmax, st)
            elif kind == "conv":
                rc = raw.qa_conv_fused_dev(ctypes.byref(payload.desc), st)
            elif kind == "conv_input":
                qp = self.c.qparams[self.graph.inputs[0].name]
                rc = raw.qa_conv_input_fused_dev(ctypes.byref(payload.desc),
                                                 self.x_dev.data_ptr(), self.in_shape[1],
                                                 float(qp.scale), qp.qmin, qp.qmax, st)
            elif kind == "rescale":
                concat, idx, src, dst = payload
                m, s = concat._mult[idx]
                qp, o = concat.in_qp[idx], concat.out_qp[0]
                rows = src.N * src.H * src.W
                rc = raw.qa_rescale_bytes_dev(src.ptr, src.pix_stride, int(src.signed), dst.ptr,
                                              dst.pix_stride, rows, src.C,
                                              int(concat.same_grid(idx)), qp.zp, m, s, o.zp,
                                              o.qmin, o.qmax, st)
            elif kind == "gap":
                layer, x, y, area = payload
                m, s = layer.multiplier(area)
                rc = raw.qa_gap_dev(x.ptr, x.pix_stride, int(x.signed), x.N, area, x.C,
                                    layer.in_zp, m, s, layer.out_zp, layer.out_qmin,
                                    layer.out_qmax, y.ptr, y.pix_stride, st)
            elif kind == "lut":
                layer, x, y, ldev = payload
                rc = raw.qa_lut_bytes_dev(x.ptr, x.pix_stride, int(x.signed), y.ptr,
                                          y.pix_stride, x.N * x.H * x.W, x.C,
                                          int(layer.lut_offset), ldev.data_ptr(),
                                          len(layer.lut), st)
            elif kind == "add":
                layer, a, b, y = payload
                (ma, sa), (mb, sb) = layer._mult
                qa, qb = layer.in_qp
                o = layer.out_qp[0]
                rc = raw.qa_add_bytes_dev(a.ptr, a.pix_stride, int(a.signed), b.ptr,
                                          b.pix_stride, int(b.signed), y.ptr, y.pix_stride,
                                          a.N * a.H * a.W, a.C, qa.zp, ma, sa, qb.zp, mb, sb,
                                          layer._sign, o.zp, o.qmin, o.qmax, st)
            elif kind == "bn":
                layer, x, y, (mdev, sdev, bdev) = payload
                rc = raw.qa_bn_bytes_dev(x.ptr, x.pix_stride, int(x.signed), y.ptr, y.pix_stride,
                                         x.N * x.H * x.W, x.C, layer.in_zp, mdev.data_ptr(),
                                         sdev.data_ptr(), bdev.data_ptr(), layer.out_zp,
                                         layer.out_qmin, layer.out_qmax, st)
            elif kind == "mul":
                layer, a, b, y = payload
                qa, qb = layer.in_qp
                o = layer.out_qp[0]
                rc = raw.qa_mul_bytes_dev(a.ptr, a.pix_stride, int(a.signed), b.ptr,
                                          b.pix_stride, int(b.signed), y.ptr, y.pix_stride,
                                          a.N * a.H * a.W, a.C, qa.zp, qb.zp, layer._mult,
                                          layer._shift, o.zp, o.qmin, o.qmax, st)
            elif kind == "maxpool":
                layer, x, y = payload
                from quantanything_b200.float_ops import pool_geometry

                k, s_, dl, pd = pool_geometry(layer.node, (x.N, x.C, x.H, x.W))
                rc = raw.qa_maxpool_bytes_dev(x.ptr, x.pix_stride, int(x.signed), y.ptr,
                                              y.pix_stride, x.N, x.H, x.W, x.C, k[0], k[1],
                                              s_[0], s_[1], pd[0], pd[1], dl[0], dl[1], y.H,
                                              y.W, layer.in_qmin, st)
            elif kind == "window":
                layer, x, y, geom, fill = payload
                rc = raw.qa_window_copy_bytes_dev(x.ptr, y.ptr, y.pix_stride, y.N, y.C, y.H, y.W,
                                                  geom[0].ctypes.data, geom[1].ctypes.data,
                                                  geom[2].ctypes.data, geom[3].ctypes.data,
                                                  fill, st)
            elif kind == "softmax":
                layer, x = payload
                qi, o = layer.in_qp[0], layer.out_qp[0]
                rc = raw.qa_softmax_dev(x.ptr, x.pix_stride, int(x.signed), x.N, x.C,
                                        float(qi.scale), qi.zp, float(o.scale), o.zp, o.qmin,
                                        o.qmax, self.out_q.data_ptr(), self.out_f32.data_ptr(),
                                        float(o.scale), o.zp, st)
            else:
                rc = self._launch_step(kind, payload, raw, st)
            _check(self.lib, rc, f"{kind} step")
            if on_step is not None:
                on_step(n)
            n += 1
        self.launch_count = n
        return n

    def _launch_step(self, kind, payload, raw, st):
        """Launch of a step kind this class does not plan (subclasses)."""
        raise AssertionError(kind)

    def forward_device(self, x=None):
        """Enqueues the whole forward on the current stream (eagerly, no graph).

        ``x``: optional float32 device tensor [N, C, H, W] copied into the
        input buffer first.  Returns the float32 device output."""
        if x is not None:
            self.x_dev.copy_(x)
        self._launch_all(torch.cuda.current_stream(self.device).cuda_stream)
        return self.out_f32

    def forward_traced(self, x=None):
        """forward_device with one NVTX range per launch, named
        ``step <i>: <layer label>`` (the labels of step_costs), so that a
        profiler can attribute kernels to layers (``ncu --nvtx
        --nvtx-include "step 3: *"`` captures one layer)."""
        nvtx = torch.cuda.nvtx
        labels = [c[0] for c in self.step_costs()]
        if x is not None:
            self.x_dev.copy_(x)

        def mark(i):
            nvtx.range_pop()
            if i + 1 < len(labels):
                nvtx.range_push(f"step {i + 1}: {labels[i + 1]}")

        nvtx.range_push(f"step 0: {labels[0]}")
        self._launch_all(torch.cuda.current_stream(self.device).cuda_stream, on_step=mark)
        return self.out_f32

    def capture(self):
        """Captures the forward in a CUDA graph (after one eager warm-up)."""
        torch.cuda.synchronize(self.device)
        self.forward_device()
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(self.device)
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self._launch_all(s.cuda_stream)
        torch.cuda.synchronize(self.device)
        self._graph = g
        return g

    def replay(self):
        """Replays the captured forward on the current stream."""
        if self._graph is None:
            self.capture()
        self._graph.replay()
        return self.out_f32

    def check_status(self):
        """Raises if any kernel reported a bounded-wait timeout.  A forward
        that stopped early may leave the fused pooling's running sums
        partly filled: they are zeroed again before the error is raised."""
        rc = self.lib.raw.qa_device_status_dev(
            ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
        if rc != 0:
            for t in getattr(self, "_gap_scratch", []):
                t.zero_()
        _check(self.lib, rc, "device status")

    def run_async(self, x_pinned, out_pinned):
        """Enqueues host->device copy, the captured forward and the copy of
        the float32 output back to ``out_pinned`` on the current stream."""
        self.x_dev.copy_(x_pinned, non_blocking=True)
        y = self.replay()
        out_pinned.copy_(y, non_blocking=True)
        return out_pinned

    def run_pipelined(self, xs_pinned, outs_pinned, collect=None):
        """Host-to-host forwards of a sequence of pinned float32 batches, each
        batch's host->device copy overlapped with the previous batch's
        forward: the copies run on a side stream into two alternating staging
        buffers; the current stream waits for its batch, moves it into the
        input buffer (device to device), replays the captured forward and
        copies the float32 result into ``outs_pinned[i]``.  Everything is
        enqueued; the outputs are valid after the current stream
        synchronizes.

        ``collect``: optional callable applied to each batch's float32 device
        output before the copy to the host (for example the multi-GPU
        all-gather of every rank's shard, ``distributed.gather_outputs_device``);
        ``outs_pinned[i]`` then receives what it returns."""
        if len(xs_pinned) != len(outs_pinned):
            raise ValueError("one output buffer per input batch")
        comp = torch.cuda.current_stream(self.device)
        if getattr(self, "_copy_stream", None) is None:
            self._copy_stream = torch.cuda.Stream(self.device)
            self._staging = [torch.empty_like(self.x_dev) for _ in range(2)]
            self._copied = [torch.cuda.Event() for _ in range(2)]
            self._consumed = [torch.cuda.Event() for _ in range(2)]
        cs = self._copy_stream
        start = torch.cuda.Event()
        start.record(comp)
        cs.wait_event(start)  # nothing of this call starts before the caller's work
        for i, (x, out) in enumerate(zip(xs_pinned, outs_pinned)):
            b = i % 2
            with torch.cuda.stream(cs):
                if i >= 2:
                    cs.wait_event(self._consumed[b])  # staging b was moved out
                self._staging[b].copy_(x, non_blocking=True)
                self._copied[b].record(cs)
            comp.wait_event(self._copied[b])
            self.x_dev.copy_(self._staging[b], non_blocking=True)
            self._consumed[b].record(comp)
            y = self.replay()
            if collect is not None:
                y = collect(y)
            out.copy_(y, non_blocking=True)
        return outs_pinned

    def run(self, x_host, out=None):
        """Public host-to-host call: copies ``x_host`` (float32 NCHW) in,
        runs the captured forward, returns the float32 output on the host."""
        xs = torch.as_tensor(np.ascontiguousarray(x_host, dtype=np.float32))
        if tuple(xs.shape) != self.in_shape:
            raise ValueError(f"input shape {tuple(xs.shape)} != planned {self.in_shape}")
        self.x_dev.copy_(xs, non_blocking=xs.is_pinned())
        y = self.replay()
        host = out if out is not None else torch.empty(y.shape, dtype=torch.float32,
                                                       pin_memory=True)
        host.copy_(y, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return host.numpy()

    def tensor(self, name):
        """A planned tensor as int32 NCHW (inspection helper; copies)."""
        v = self._views[name]
        rows = v.N * v.H * v.W
        t = torch.as_strided(v.buf, (rows, v.C), (v.pix_stride, 1), v.offset)
        t = (t.view(torch.int8) if v.signed else t).to(torch.int32)
        return t.reshape(v.N, v.H, v.W, v.C).permute(0, 3, 1, 2).contiguous()

    def output_int(self):
        """int32 graph output (before the final dequantize) of the last run."""
        return self.out_q

    def output_qparams(self):
        """QParams of the graph output (the grid ``output_int`` is on)."""
        return self.c.qparams[self.graph.outputs[0]]


def make_resident(container, batch, device=None):
    """The device-resident executor that runs ``container``'s graph: a
    transformer graph (LayerNormalization present) on ResidentViT (int16:
    ResidentViT16), int16 and
    uint8 graphs on ResidentNet16 (byte-split contractions; uint8 weights
    are asymmetric and exceed int8), other 8-bit graphs on ResidentNet.
    Raises UnsupportedGraph when none of them covers the graph."""
    from quantanything_b200.resident16 import ResidentNet16
    from quantanything_b200.resident_vit import ResidentViT

    from quantanything_b200.resident_vit import ResidentViT16

    layer0 = container.layers[0]
    if any(n.op_type == "LayerNormalization" for n in container.graph.nodes):
        if layer0.num_bits == 16:
            return ResidentViT16(container, batch, device)
        return ResidentViT(container, batch, device)
    if layer0.num_bits == 16 or (layer0.num_bits == 8 and not layer0.signed):
        return ResidentNet16(container, batch, device)
    return ResidentNet(container, batch, device)
