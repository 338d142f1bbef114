"""Device-resident integer inference of Vision Transformer graphs.

The graphs are the reference's ViT after its load-time passes (the form
``networks.vit`` builds): patch-embedding Conv, class token + positional
embedding, pre-LN blocks of multi-head self-attention and a GELU MLP, the
class token gathered before the final LayerNorm, a Gemm head.  Activations
stay on the device as byte rows [tokens, features]:

* every weighted layer (patch Conv, QKV / projection / MLP MatMuls, head
  Gemm) runs on the tcgen05 fused-contraction kernel, with the GELU table
  and the residual Add fused into its epilogue;
* Concat(class token) + Add(positions) is one kernel of exact integer
  tables (``qa_vit_embed_dev``);
* LayerNorm (``qa_layernorm_bytes_dev``) and the attention core —
  scores MatMul, the 1/sqrt(head_dim) Mul, Softmax and the MatMul with V,
  each a float fallback of the reference (quant_layers.py:195-205) —
  (``qa_attention_bytes_dev``, one CTA per image and head) reproduce the
  reference's dequantize -> float -> quantize arithmetic;
* the class-token Gather is a row gather through its requantization table.

The float fallbacks match the reference within one output step (the
tolerance stated for them): their sums run in a different order than
NumPy's.
"""
import ctypes

import numpy as np
import torch

from quantanything_b200.layers import (ActivationQuantize, AddQuantize, BaseQuantLayer,
                                       ConcatQuantize, ConvQuantize, GemmQuantize, MulQuantize,
                                       ShapingQuantize)
from quantanything_b200.resident import ResidentNet, UnsupportedGraph, View, _round_up
from quantanything_b200.resident16 import (UINT16_SHIFT, ResidentNet16, device_api16,
                                          shifted_container)

_I32_MIN, _I32_MAX = -(1 << 31), (1 << 31) - 1
_TAB = np.arange(-128, 256, dtype=np.int64)  # byte-domain table index v + 128


class ResidentViT(ResidentNet):
    """Fused device-resident integer inference of a ViT graph (8-bit)."""

    _domain = _TAB  # every activation value, in table-index order

    def __init__(self, container, batch, device=None):
        super().__init__(container, batch, device, fuse_input=False)

    # ---------------------------------------------------------------- plan --
    def _row_view(self, rows, C, qp, pix_stride=None):
        stride = pix_stride or _round_up(C, 16)
        return View(self._alloc(rows * stride), 0, stride, rows, 1, 1, C, self.signed, qp)

    def _input_view(self, N, H, W, C, stride, qp):
        return View(self._alloc(N * H * W * stride), 0, stride, N, H, W, C, self.signed, qp)

    def _cls_row_dev(self, cls_row):
        return self._dev(cls_row.astype(np.int64) & 0xFF, np.uint8)

    def _plan(self):
        g, c = self.graph, self.c
        layers = {l.name: l for l in c.layers}
        self._layers = layers
        consumers = {}
        for node in g.nodes:
            for i in node.inputs:
                if i:
                    consumers.setdefault(i, []).append(node)
        self._consumers = consumers
        self._concat_slot, self._concat_done, self._producer_step = {}, {}, {}
        self._transposed = {}  # transposed token rows read in place by MatMuls
        in_name = g.inputs[0].name
        shp = g.inputs[0].shape
        if int(shp[0]) != self.batch:
            raise UnsupportedGraph(f"the ViT graph is built for batch {shp[0]}")
        self.in_shape = (self.batch, int(shp[1]), int(shp[2]), int(shp[3]))
        Cin = self.in_shape[1]
        qp_in = c.qparams[in_name]
        stride_in = _round_up(Cin, 4)
        self._views = {in_name: self._input_view(self.batch, self.in_shape[2], self.in_shape[3],
                                                 Cin, stride_in, qp_in)}
        self._in_view = self._views[in_name]
        self.x_dev = torch.empty(self.in_shape, dtype=torch.float32, device=self.device)
        self.steps.append(("quantize", in_name))
        self._shapes = {in_name: self.in_shape}
        fused_away = set()
        attention = self._find_attention(g, layers)
        for node in g.nodes:
            if node.name in fused_away:
                continue
            layer = layers[node.name]
            op = node.op_type
            if isinstance(layer, ConvQuantize):
                if node.inputs[0] != in_name:
                    raise UnsupportedGraph("only the patch embedding may be a Conv")
                P = self._patch_rows(layer)
                if P:
                    # the input quantizer writes the conv's im2col rows; the
                    # conv runs as a row-matrix GEMM over them
                    v = self._in_view
                    N, _, H, W = self.in_shape
                    K = P * P * 4
                    pv = View(v.buf, 0, K, N, H // P, W // P, K, v.signed, v.qp)
                    self._views[in_name] = self._in_view = pv
                    self._in_patch = P
                self._plan_contraction(layer, layers, fused_away, patch=P)
            elif (op == "Transpose" and node.outputs[0] not in attention["all"]
                  and node.inputs[0] != getattr(self, "_token_pending", None)):
                self._plan_transposed_tokens(node)
            elif op in ("Reshape", "Transpose") and node.outputs[0] not in attention["all"]:
                self._plan_token_alias(node)
            elif (op == "MatMul" and type(layer) is BaseQuantLayer
                  and node.outputs[0] not in attention["all"]):
                self._plan_matmul_act(layer)
            elif isinstance(layer, ConcatQuantize):
                self._plan_embed(layer, layers, fused_away)
            elif op == "LayerNormalization":
                self._plan_layernorm(layer)
            elif isinstance(layer, GemmQuantize):
                x = self._views[node.inputs[0]]
                self._shapes[node.inputs[0]] = (x.N, x.C, 1, 1)
                self._plan_contraction(layer, layers, fused_away)
                produced = self._last_produced()
                y = self._views[produced]
                self._shapes[produced] = (y.N, y.C, 1, 1)
            elif node.name in attention["emit"]:
                self._plan_attention(attention["emit"][node.name], layers)
            elif node.outputs[0] in attention["all"]:
                continue  # inside an attention block: planned with it
            elif op == "Gather":
                self._plan_gather(layer)
            else:
                raise UnsupportedGraph(f"{op} ({node.name}) has no resident ViT kernel")
        out = g.outputs[0]
        if out not in self._views:
            raise UnsupportedGraph("graph output not produced")
        y = self._views[out]
        N, C = y.N, y.C
        self.out_q = torch.empty((N, C), dtype=torch.int32, device=self.device)
        self.out_f32 = torch.empty((N, C), dtype=torch.float32, device=self.device)
        self._outputs_f32 = {out: self.out_f32}
        self.steps.append(("dequant", (y, c.qparams[out])))

    def _patch_rows(self, layer):
        """Patch size P when the patch embedding is a P x P, stride-P conv
        without padding or dilation that the input quantizer can write as
        im2col rows (qa_quantize_to_patch_rows_dev), else 0."""
        N, C, H, W = self.in_shape
        kh, kw = (int(v) for v in layer.w_q.shape[2:])
        strides, pads, dil, groups = layer.geometry((N, C, H, W))
        if (kh != kw or tuple(strides) != (kh, kw) or any(pads) or tuple(dil) != (1, 1)
                or groups != 1 or C > 4 or kh % 4 or H % kh or W % kw or W % 4):
            return 0
        return kh

    def _last_produced(self):
        step = self.steps[-1][1]
        return [k for k, v in self._producer_step.items() if v is step][-1]

    def _plan_token_alias(self, node):
        """Reshape / Transpose of the patch grid into token rows: the NHWC
        patch-embedding output already is [B, tokens, D] in memory."""
        x = self._views[node.inputs[0]]
        if node.op_type == "Reshape":
            shape = [int(v) for v in np.asarray(self.graph.initializers[node.inputs[1]]).ravel()]
            if len(shape) != 3 or shape[0] != self.batch or shape[1] != x.C:
                raise UnsupportedGraph(f"{node.name}: unexpected patch reshape {shape}")
            self._views[node.outputs[0]] = x
            self._token_pending = node.outputs[0]
        else:
            if node.attr("perm") != [0, 2, 1] or node.inputs[0] != getattr(self, "_token_pending",
                                                                           None):
                raise UnsupportedGraph(f"{node.name}: unexpected transpose")
            rows = x.N * x.H * x.W
            self._views[node.outputs[0]] = View(x.buf, x.offset, x.pix_stride, rows, 1, 1, x.C,
                                                x.signed, x.qp, x.plane)
            self._tokens_per_image = x.H * x.W

    def _plan_transposed_tokens(self, node):
        """Transpose(perm [0, 2, 1]) of token rows [B, T, D] read only by
        activation x activation MatMuls: no kernel, the MatMul reads the
        rows with its strides swapped."""
        x = self._views[node.inputs[0]]
        readers = self._consumers.get(node.outputs[0], [])
        if (node.attr("perm") != [0, 2, 1] or not readers
                or any(r.op_type != "MatMul" or r.inputs[1] != node.outputs[0]
                       for r in readers)):
            raise UnsupportedGraph(f"{node.name}: only a [0, 2, 1] Transpose read as the "
                                   "second operand of MatMuls is resident")
        self._transposed[node.outputs[0]] = x

    def _plan_matmul_act(self, layer):
        """MatMul of two activations [B, M, K] x [B, K, N] (the reference's
        float fallback, quant_layers.py:195-205): one qa_matmul_act_bytes_dev
        launch over the token rows; a [0, 2, 1]-transposed second operand is
        read in place."""
        node = layer.node
        a = self._views[node.inputs[0]]
        Bn = self.batch
        if len(node.inputs) > 2 and node.inputs[2] or a.N % Bn:
            raise UnsupportedGraph(f"{node.name}: MatMul of [B, M, K] token rows expected")
        M, K = a.N // Bn, a.C
        if node.inputs[1] in self._transposed:
            bt = self._transposed[node.inputs[1]]
            if bt.C != K or bt.N % Bn:
                raise UnsupportedGraph(f"{node.name}: operand shapes do not match")
            N = bt.N // Bn
            bview, strides = bt, (N * bt.pix_stride, 1, bt.pix_stride)   # b_sb, b_sk, b_sn
        else:
            bv = self._views[node.inputs[1]]
            if bv.N != Bn * K:
                raise UnsupportedGraph(f"{node.name}: operand shapes do not match")
            N = bv.C
            bview, strides = bv, (K * bv.pix_stride, bv.pix_stride, 1)
        y = self._row_view(Bn * M, N, layer.out_qp[0])
        self._views[node.outputs[0]] = y
        self.steps.append(("matmul_act", (layer, a, bview, y, M, N, K, strides)))

    def _plan_embed(self, concat, layers, fused_away):
        """Concat(class token, patch tokens) -> Add(positions) as one table
        kernel; the tables come from the reference's integer functions (the
        library's qa_rescale), so the result is exact."""
        node = concat.node
        c, lib = self.c, self.lib
        cls_name, x_name = node.inputs
        if node.attr("axis") != 1 or not self.graph.is_constant(cls_name):
            raise UnsupportedGraph("embedding Concat: expected (constant class token, tokens)")
        add = self._only_consumer(node.outputs[0])
        if add is None or not isinstance(layers[add.name], AddQuantize):
            raise UnsupportedGraph("embedding Concat must feed the positional Add")
        al = layers[add.name]
        if add.inputs[0] != node.outputs[0] or not self.graph.is_constant(add.inputs[1]):
            raise UnsupportedGraph("positional Add: expected (tokens, constant)")
        x = self._views[x_name]
        T = self._tokens_per_image + 1
        D = x.C
        o = concat.out_qp[0]

        def concat_rescale(v, idx):
            qp = concat.in_qp[idx]
            if concat.same_grid(idx):
                return np.clip(v, o.qmin, o.qmax).astype(np.int64)
            m, s = concat._mult[idx]
            return lib.rescale(np.asarray(v, np.int32), qp.zp, m, s, o.zp, o.qmin,
                               o.qmax).astype(np.int64)

        (ma, sa), (mb, sb) = al._mult
        qa, qb = al.in_qp
        ao = al.out_qp[0]

        def term(v, z, m, s):  # mbqm(v - z, m, s), unclamped
            return lib.rescale(np.asarray(v, np.int32), z, m, s, 0, _I32_MIN,
                               _I32_MAX).astype(np.int64)

        ta = term(concat_rescale(self._domain, 1), qa.zp, ma, sa)
        pos_q = np.asarray(c._const_q[add.inputs[1]], np.int64).reshape(T, D)
        pos = al._sign * term(pos_q, qb.zp, mb, sb) + ao.zp
        cls_q = np.asarray(c._const_q[cls_name], np.int64).reshape(-1, D)[0]
        cls_row = np.clip(term(concat_rescale(cls_q, 0), qa.zp, ma, sa) + pos[0], ao.qmin,
                          ao.qmax)
        y = self._row_view(self.batch * T, D, ao)
        self._views[add.outputs[0]] = y
        fused_away.add(add.name)
        self.steps.append(("vit_embed", (x, y, T, D, ao,
                                         self._dev(ta, np.int32), self._dev(pos, np.int32),
                                         self._cls_row_dev(cls_row))))

    def _plan_layernorm(self, layer):
        node = layer.node
        x = self._views[node.inputs[0]]
        D = x.C
        gamma = np.asarray(self.graph.initializers[node.inputs[1]], np.float32).reshape(-1)
        beta = (np.asarray(self.graph.initializers[node.inputs[2]], np.float32).reshape(-1)
                if len(node.inputs) > 2 and node.inputs[2] else None)
        axis = node.attr("axis", -1)
        if axis not in (-1, len(self._dims(node.inputs[0])) - 1) or gamma.size != D:
            raise UnsupportedGraph(f"{node.name}: LayerNorm over the feature axis only")
        y = self._row_view(x.N, D, layer.out_qp[0])
        self._views[node.outputs[0]] = y
        self.steps.append(("layernorm", (layer, x, y, self._dev(gamma, np.float32),
                                         None if beta is None else self._dev(beta, np.float32),
                                         float(node.attr("epsilon", 1e-5)))))

    def _dims(self, name):
        v = self._views[name]
        return (v.N, v.C)

    def _plan_gather(self, layer):
        node = layer.node
        x = self._views[node.inputs[0]]
        idx = np.asarray(self.graph.initializers.get(node.inputs[1])).reshape(-1)
        if node.attr("axis", 0) != 1 or idx.size != 1:
            raise UnsupportedGraph(f"{node.name}: expected one token gathered along axis 1")
        T = x.N // self.batch
        first = int(idx[0]) % T
        # the Gather's requantization (dequantize -> take -> quantize) per byte
        table = layer.quantized_infer_integer(
            [self._domain.reshape(1, 1, -1).astype(np.int32)])[0]
        table = np.asarray(table, np.int64).reshape(-1)
        y = self._row_view(self.batch, x.C, layer.out_qp[0])
        self._views[node.outputs[0]] = y
        self.steps.append(("gather", (x, y, T, first, self._dev(table, np.int32))))

    # ----------------------------------------------------------- attention --
    def _find_attention(self, g, layers):
        """The nodes of every attention block: from the QKV projection's
        output through Reshape / Transpose / Split / Squeeze, the scores
        MatMul, the scale Mul, Softmax, the MatMul with V, to the head-merge
        Transpose + Reshape."""
        producers = {o: n for n in g.nodes for o in n.outputs}
        emit, every = {}, set()
        for sm in [n for n in g.nodes if n.op_type == "Softmax"]:
            mul = producers[sm.inputs[0]]
            mm1 = producers[[i for i in mul.inputs if not g.is_constant(i)][0]]
            const = [i for i in mul.inputs if g.is_constant(i)]
            if mul.op_type != "Mul" or mm1.op_type != "MatMul" or len(const) != 1:
                raise UnsupportedGraph("attention: expected MatMul -> Mul(constant) -> Softmax")
            q_sq = producers[mm1.inputs[0]]
            kt = producers[mm1.inputs[1]]
            k_sq = producers[kt.inputs[0]]
            (mm2,) = self._consumers[sm.outputs[0]]
            v_sq = producers[mm2.inputs[1]]
            split = producers[q_sq.inputs[0]]
            tr = producers[split.inputs[0]]
            rs = producers[tr.inputs[0]]
            (tr2,) = self._consumers[mm2.outputs[0]]
            (rs2,) = self._consumers[tr2.outputs[0]]
            nodes = [rs, tr, split, q_sq, k_sq, v_sq, kt, mm1, mul, sm, mm2, tr2, rs2]
            ok = (rs.op_type == "Reshape" and tr.op_type == "Transpose"
                  and tr.attr("perm") == [2, 0, 3, 1, 4] and split.op_type == "Split"
                  and all(n.op_type == "Squeeze" for n in (q_sq, k_sq, v_sq))
                  and kt.op_type == "Transpose" and kt.attr("perm") == [0, 1, 3, 2]
                  and [producers[n.inputs[0]] for n in (q_sq, k_sq, v_sq)] == [split] * 3
                  and [q_sq.inputs[0], k_sq.inputs[0], v_sq.inputs[0]] == list(split.outputs)
                  and mm2.op_type == "MatMul" and tr2.op_type == "Transpose"
                  and tr2.attr("perm") == [0, 2, 1, 3] and rs2.op_type == "Reshape")
            if not ok:
                raise UnsupportedGraph("attention block does not have the expected form")
            shape = [int(v) for v in np.asarray(g.initializers[rs.inputs[1]]).ravel()]
            info = {"qkv": rs.inputs[0], "shape": shape, "mm1": mm1, "mul": mul, "sm": sm,
                    "mm2": mm2, "out": rs2.outputs[0], "scale": const[0]}
            emit[rs2.name] = info
            for n in nodes:
                every.update(n.outputs)
        return {"emit": emit, "all": every}

    def _plan_attention(self, info, layers):
        c, lib = self.c, self.lib
        qkv = self._views[info["qkv"]]
        B, T, three, H, hd = info["shape"]
        if three != 3 or B != self.batch or B * T != qkv.N or qkv.C != 3 * H * hd:
            raise UnsupportedGraph("attention: QKV shape mismatch")
        S, mul, sm, O = (layers[info[k].name] for k in ("mm1", "mul", "sm", "mm2"))
        if not isinstance(mul, MulQuantize) or not all(
                type(l) is BaseQuantLayer for l in (S, sm, O)):
            raise UnsupportedGraph("attention: unexpected layer types")
        qs, qm, qp_, qo = S.out_qp[0], mul.out_qp[0], sm.out_qp[0], O.out_qp[0]
        # Mul by the constant, as the reference's integer op, per S byte
        data_idx = [i for i, n in enumerate(mul.node.inputs) if n != info["scale"]][0]
        cq = np.asarray(c._const_q[info["scale"]], np.int32).reshape(-1)[0]
        args = [None, None]
        args[data_idx] = _TAB.astype(np.int32)
        args[1 - data_idx] = np.full(_TAB.shape, cq, np.int32)
        mul_table = np.asarray(mul.quantized_infer_integer(args)[0], np.int64)
        y = self._row_view(qkv.N, H * hd, qo)
        self._views[info["out"]] = y
        s_par = np.array([qs.scale, qm.scale, qp_.scale, qo.scale], np.float64)
        z_par = np.array([qs.zp, qs.qmin, qs.qmax, qp_.zp, qp_.qmin, qp_.qmax, qo.zp, qo.qmin,
                          qo.qmax, qm.zp], np.int64)
        p_signed = int(qp_.qmin < 0)
        # s_par / z_par are read by the host entry point: host arrays
        self.steps.append(("attention", (qkv, y, T, H, hd, s_par, z_par,
                                         self._dev(mul_table, np.int32), p_signed)))

    # -------------------------------------------------------------- launch --
    def _launch_step(self, kind, payload, raw, st):
        if kind == "vit_embed":
            x, y, T, D, ao, ta, pos, cls_row = payload
            return raw.qa_vit_embed_dev(x.ptr, x.pix_stride, int(x.signed), ta.data_ptr(),
                                        pos.data_ptr(), cls_row.data_ptr(), ao.qmin, ao.qmax,
                                        y.ptr, y.pix_stride, self.batch, T, D, st)
        if kind == "layernorm":
            layer, x, y, gamma, beta, eps = payload
            qi, o = layer.in_qp[0], layer.out_qp[0]
            return raw.qa_layernorm_bytes_dev(x.ptr, x.pix_stride, int(x.signed), qi.zp,
                                              float(qi.scale), gamma.data_ptr(),
                                              None if beta is None else beta.data_ptr(), eps,
                                              float(o.scale), o.zp, o.qmin, o.qmax, y.ptr,
                                              y.pix_stride, x.N, x.C, st)
        if kind == "attention":
            qkv, y, T, H, hd, s_par, z_par, mul_table, p_signed = payload
            qp = qkv.qp
            return raw.qa_attention_bytes_dev(qkv.ptr, qkv.pix_stride, int(qkv.signed), qp.zp,
                                              float(qp.scale), self.batch, T, H, hd,
                                              s_par.ctypes.data, z_par.ctypes.data,
                                              mul_table.data_ptr(), p_signed, y.ptr,
                                              y.pix_stride, st)
        if kind == "matmul_act":
            layer, a, b, y, M, N, K, (b_sb, b_sk, b_sn) = payload
            qa, qb = layer.in_qp[0], layer.in_qp[1]
            o = layer.out_qp[0]
            return raw.qa_matmul_act_bytes_dev(a.ptr, int(a.signed), M * a.pix_stride,
                                               a.pix_stride, 1, qa.zp, float(qa.scale), b.ptr,
                                               int(b.signed), b_sb, b_sk, b_sn, qb.zp,
                                               float(qb.scale), y.ptr, y.pix_stride, self.batch,
                                               M, N, K, float(o.scale), o.zp, o.qmin, o.qmax, st)
        if kind == "gather":
            x, y, T, first, table = payload
            return raw.qa_gather_table_dev(x.ptr, x.pix_stride, int(x.signed), T, first,
                                           table.data_ptr(), y.ptr, y.pix_stride, y.N, y.C, st)
        if kind == "dequant":
            y, qp = payload
            return raw.qa_dequantize_rows_dev(y.ptr, y.pix_stride, int(y.signed), qp.zp,
                                              float(qp.scale), self.out_q.data_ptr(),
                                              self.out_f32.data_ptr(), y.N, y.C, st)
        raise AssertionError(kind)

    def step_costs(self):
        costs = []
        for kind, payload in self.steps:
            if kind in ("quantize", "conv"):
                costs.extend(ResidentNet.step_costs(_Only(self, kind, payload)))
            elif kind == "attention":
                qkv, y, T, H, hd = payload[:5]
                costs.append((f"attention {self.batch}x{H} heads T={T} hd={hd}",
                              qkv.N * qkv.C + y.N * y.C, 4 * self.batch * H * T * T * hd))
            elif kind == "dequant":
                y = payload[0]
                costs.append((kind, y.N * y.C * 9, 0))
            elif kind == "matmul_act":
                layer, a, b, y, M, N, K = payload[:7]
                costs.append((f"matmul act x act {self.batch}x{M}x{K}x{N}",
                              self.batch * (M * K + K * N + M * N),
                              2 * self.batch * M * N * K))
            else:
                x, y = (payload[1], payload[2]) if kind == "layernorm" else payload[:2]
                costs.append((kind, x.N * x.C + y.N * y.C, 0))
        return costs


class _Only:
    """A view of one step for ResidentNet.step_costs."""

    def __init__(self, net, kind, payload):
        self.steps = [(kind, payload)]
        self.in_shape = net.in_shape
        self._in_view = net._in_view
        self._in_patch = net._in_patch


class ResidentViT16(ResidentViT, ResidentNet16):
    """Device-resident integer inference of an int16 ViT graph (the
    reference's accurate ViT route, README.md:130-135).

    Activations are int16 tensors in two byte planes (the 16-bit executor's
    layout): the patch embedding, QKV / projection / MLP MatMuls (GELU table
    and residual Add fused) and the head run on the byte-split tensor-core
    kernel with its exact int64 combine; the token embedding, the
    class-token Gather, LayerNorm, the attention core and the output
    dequantize run on the 16-bit plane kernels (qa_*16_dev), with the same
    float-fallback arithmetic as the 8-bit route.  uint16 graphs run here too,
    their activations held 32768 lower (``resident16.shifted_container``)
    and their 17-bit centred weights in three byte planes."""

    _domain = np.arange(-32768, 32768, dtype=np.int64)

    def __init__(self, container, batch, device=None):
        self._planes = []
        self._lut16 = {}
        # uint16: activations held 32768 lower in the signed planes (every
        # activation zero point, range, table and quantized constant moved
        # with them) and the 17-bit centred weights in three byte planes, as
        # in ResidentNet16
        layer0 = container.layers[0]
        self._orig = container
        self._act_shift = UINT16_SHIFT if (layer0.num_bits == 16 and not layer0.signed) else 0
        self._w_planes = 3 if self._act_shift else 2
        if self._act_shift:
            container = shifted_container(container, self._act_shift)
        ResidentNet.__init__(self, container, batch, device, fuse_input=False)
        device_api16(self.lib)
        vit16_api(self.lib)
        self._descs = {}

    def _row_view(self, rows, C, qp, pix_stride=None):
        return self._new_view(rows, 1, 1, C, qp, pix_stride)

    def _input_view(self, N, H, W, C, stride, qp):
        return self._new_view(N, H, W, C, qp, pix_stride=stride)

    def _cls_row_dev(self, cls_row):
        return self._dev(cls_row, np.int32)

    def _patch_rows(self, layer):
        return 0  # the patch embedding gathers 4-byte taps from the int16 planes

    def _plan_matmul_act(self, layer):
        raise UnsupportedGraph(f"{layer.name}: activation x activation MatMul of 16-bit "
                               "tensors has no resident kernel")

    def _plan_attention(self, info, layers):
        c = self.c
        qkv = self._views[info["qkv"]]
        B, T, three, H, hd = info["shape"]
        if three != 3 or B != self.batch or B * T != qkv.N or qkv.C != 3 * H * hd:
            raise UnsupportedGraph("attention: QKV shape mismatch")
        S, mul, sm, O = (layers[info[k].name] for k in ("mm1", "mul", "sm", "mm2"))
        if not isinstance(mul, MulQuantize) or not all(
                type(l) is BaseQuantLayer for l in (S, sm, O)):
            raise UnsupportedGraph("attention: unexpected layer types")
        qs, qm, qp_, qo = S.out_qp[0], mul.out_qp[0], sm.out_qp[0], O.out_qp[0]
        data_idx = [i for i, n in enumerate(mul.node.inputs) if n != info["scale"]][0]
        qd, qc = mul.in_qp[data_idx], mul.in_qp[1 - data_idx]
        cq = int(np.asarray(c._const_q[info["scale"]], np.int64).reshape(-1)[0])
        y = self._row_view(qkv.N, H * hd, qo)
        self._views[info["out"]] = y
        s_par = np.array([qs.scale, qm.scale, qp_.scale, qo.scale], np.float64)
        z_par = np.array([qs.zp, qs.qmin, qs.qmax, qm.zp, qm.qmin, qm.qmax, qp_.zp, qp_.qmin,
                          qp_.qmax, qo.zp, qo.qmin, qo.qmax], np.int64)
        mul_par = np.array([cq, qc.zp, qd.zp, int(mul._mult), int(mul._shift)], np.int64)
        self.steps.append(("attention", (qkv, y, T, H, hd, s_par, z_par, mul_par)))

    def _launch_step(self, kind, payload, raw, st):
        if kind == "vit_embed":
            x, y, T, D, ao, ta, pos, cls_row = payload
            return raw.qa_vit_embed16_dev(x.ptr, x.plane, x.pix_stride, ta.data_ptr(),
                                          pos.data_ptr(), cls_row.data_ptr(), ao.qmin, ao.qmax,
                                          y.ptr, y.plane, y.pix_stride, self.batch, T, D, st)
        if kind == "layernorm":
            layer, x, y, gamma, beta, eps = payload
            qi, o = layer.in_qp[0], layer.out_qp[0]
            return raw.qa_layernorm16_dev(x.ptr, x.plane, x.pix_stride, qi.zp, float(qi.scale),
                                          gamma.data_ptr(),
                                          None if beta is None else beta.data_ptr(), eps,
                                          float(o.scale), o.zp, o.qmin, o.qmax, y.ptr, y.plane,
                                          y.pix_stride, x.N, x.C, st)
        if kind == "attention":
            qkv, y, T, H, hd, s_par, z_par, mul_par = payload
            qp = qkv.qp
            return raw.qa_attention16_dev(qkv.ptr, qkv.plane, qkv.pix_stride, qp.zp,
                                          float(qp.scale), self.batch, T, H, hd,
                                          s_par.ctypes.data, z_par.ctypes.data,
                                          mul_par.ctypes.data, y.ptr, y.plane, y.pix_stride, st)
        if kind == "gather":
            x, y, T, first, table = payload
            return raw.qa_gather16_dev(x.ptr, x.plane, x.pix_stride, T, first, table.data_ptr(),
                                       y.ptr, y.plane, y.pix_stride, y.N, y.C, st)
        if kind == "dequant":
            y, qp = payload
            return raw.qa_dequantize_rows16_dev(y.ptr, y.plane, y.pix_stride, qp.zp,
                                                float(qp.scale), self.out_q.data_ptr(),
                                                self.out_f32.data_ptr(), y.N, y.C, st)
        raise AssertionError(kind)


_VIT16_SIGNATURES = {
    "qa_vit_embed16_dev": [ctypes.c_void_p] + [ctypes.c_int64] * 2 + [ctypes.c_void_p] * 3
    + [ctypes.c_int64] * 2 + [ctypes.c_void_p] + [ctypes.c_int64] * 5 + [ctypes.c_void_p],
    "qa_layernorm16_dev": [ctypes.c_void_p] + [ctypes.c_int64] * 3 + [ctypes.c_double]
    + [ctypes.c_void_p] * 2 + [ctypes.c_double] * 2 + [ctypes.c_int64] * 3 + [ctypes.c_void_p]
    + [ctypes.c_int64] * 4 + [ctypes.c_void_p],
    "qa_attention16_dev": [ctypes.c_void_p] + [ctypes.c_int64] * 3 + [ctypes.c_double]
    + [ctypes.c_int64] * 4 + [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 2 + [ctypes.c_void_p],
    "qa_gather16_dev": [ctypes.c_void_p] + [ctypes.c_int64] * 4 + [ctypes.c_void_p] * 2
    + [ctypes.c_int64] * 4 + [ctypes.c_void_p],
    "qa_dequantize_rows16_dev": [ctypes.c_void_p] + [ctypes.c_int64] * 3 + [ctypes.c_double]
    + [ctypes.c_void_p] * 2 + [ctypes.c_int64] * 2 + [ctypes.c_void_p],
}


def vit16_api(lib):
    """Declares the 16-bit transformer entry points on a loaded library."""
    raw = lib.raw
    if not getattr(raw, "_qa_vit16_declared", False):
        for name, args in _VIT16_SIGNATURES.items():
            fn = getattr(raw, name)
            fn.restype, fn.argtypes = ctypes.c_int, args
        raw._qa_vit16_declared = True
    return raw
