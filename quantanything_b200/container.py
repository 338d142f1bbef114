"""QuantContainer: calibration, q.json persistence and integer execution.

Mirrors the reference's ``quantization/quant_container.py``: same public
methods (``calibrate``, ``finalize``, ``run_graph``, ``save``, ``load``,
``layers``) and the same q.json format, so a q.json written by the
reference loads here and reproduces its integer parameters exactly.

Execution modes:
  * ``"float"``     -- float32 reference pass;
  * ``"calibrate"`` -- float pass that records per-tensor min / max;
  * ``"integer"``   -- the drop-in execution: one kernel-library call per
    layer on host int32 tensors (quant_container.py:135-193).
The device-resident, fused execution of the same prepared layers is
:class:`quantanything_b200.resident.ResidentNet`.

Multi-GPU calibration: ``calibrate(..., reduce_ranges=fn)`` lets each rank
run its shard of the calibration batches, then combines the per-tensor
ranges with ``fn`` (an all-reduce of MIN / MAX, see
:mod:`quantanything_b200.distributed`) before ``finalize``, so every rank
derives identical parameters.
"""

import json
from pathlib import Path

import numpy as np

from quantanything_b200 import float_ops, native
from quantanything_b200.layers import map_node_to_quant
from quantanything_b200.utils import QParams, calculate_scale_zp

MODES = ("float", "calibrate", "integer")


class QuantContainer:
    """Post-training static quantization of a graph (quant_container.py:27-267)."""

    def __init__(self, graph, quant_type="int8", per_channel=True, lib=None):
        self.graph = graph
        self.quant_type = quant_type
        self.per_channel = per_channel
        self._lib = lib
        self.quant_layers = {n.name: map_node_to_quant(n, graph, quant_type, per_channel, lib)
                             for n in graph.nodes}
        self.qparams = {}
        self._input_range = {}
        self._const_names = self._constant_operands()
        self._const_q = {}
        self.calibrated = False

    @property
    def lib(self):
        return self._lib if self._lib is not None else native.get_library()

    def _constant_operands(self):
        names = []
        for layer in self.quant_layers.values():
            for n in layer.data_inputs:
                if self.graph.is_constant(n) and n not in names:
                    names.append(n)
        return names

    @property
    def layers(self):
        return list(self.quant_layers.values())

    # ---------------------------------------------------------- calibration --
    def calibrate(self, x_calib, reduce_ranges=None, device=False):
        """Runs the calibration batches, combines ranges across ranks with
        ``reduce_ranges`` when given, then finalizes (quant_container.py:75-91).

        ``device=True`` runs the float pass and the range reductions on the
        GPU (``calibrate_device.calibrate_on_device``): the batches' tensors
        stay in device memory and only the range table comes back."""
        batches = [x_calib] if isinstance(x_calib, (np.ndarray, dict)) else list(x_calib)
        if not batches:
            raise ValueError("no calibration data provided")
        if device:
            from quantanything_b200.calibrate_device import calibrate_on_device

            if reduce_ranges is not None:
                raise ValueError("device calibration combines ranks with calibrate_on_device("
                                 "..., reduce_group=...)")
            calibrate_on_device(self, batches)
            return
        for batch in batches:
            self.run_graph(batch, mode="calibrate")
        if reduce_ranges is not None:
            self.set_ranges(reduce_ranges(self.get_ranges()))
        self.finalize()

    def get_ranges(self):
        """Packed ``{tensor: (lo, hi)}`` of every observed range."""
        r = {f"in:{k}": v for k, v in self._input_range.items()}
        for layer in self.layers:
            for i, name in enumerate(layer.node.outputs):
                if layer.out_min[i] is not None:
                    r[f"{layer.name}:{i}"] = (layer.out_min[i], layer.out_max[i])
        return r

    def set_ranges(self, ranges):
        for key, (lo, hi) in ranges.items():
            if key.startswith("in:"):
                self._input_range[key[3:]] = (float(lo), float(hi))
            else:
                lname, idx = key.rsplit(":", 1)
                layer = self.quant_layers[lname]
                layer.out_min[int(idx)], layer.out_max[int(idx)] = float(lo), float(hi)

    def finalize(self):
        """qparams from the collected ranges (quant_container.py:93-112)."""
        self.qparams = {name: QParams(*calculate_scale_zp(lo, hi, self.quant_type))
                        for name, (lo, hi) in self._input_range.items()}
        self._const_q = {}
        for name in self._const_names:
            value = self.graph.initializers[name].astype(np.float32)
            qp = QParams(*calculate_scale_zp(value.min(), value.max(), self.quant_type))
            self.qparams[name] = qp
            self._const_q[name] = self.lib.quantize_f32(value, qp.scale, qp.zp, qp.qmin, qp.qmax)
        for layer in self.layers:
            layer.finalize_calibration(self)
        self.calibrated = True

    # ------------------------------------------------------------ execution --
    def run_graph(self, x, mode="integer"):
        if mode not in MODES:
            raise ValueError(f"Unknown graph mode: {mode}")
        if mode == "float":
            return float_ops.run_float(self.graph, x, lib=self.lib)
        return self._execute(x, mode)

    def quantize_inputs(self, feeds):
        """Graph inputs -> int32 tensors on their input grid."""
        out = {}
        for name, value in feeds.items():
            qp = self.qparams[name]
            out[name] = self.lib.quantize_f32(value, qp.scale, qp.zp, qp.qmin, qp.qmax)
        return out

    def _execute(self, x, mode, trace=None):
        graph = self.graph
        if mode != "calibrate" and not self.calibrated:
            raise ValueError("Container is not calibrated; call calibrate().")
        feeds = float_ops.normalize_feeds(graph, x)
        env = {}
        if mode == "calibrate":
            for name, value in feeds.items():
                lo, hi = float(value.min()), float(value.max())
                cur = self._input_range.get(name)
                self._input_range[name] = (lo, hi) if cur is None else (min(cur[0], lo),
                                                                       max(cur[1], hi))
                env[name] = value
        else:
            env.update(self.quantize_inputs(feeds))
        for name in self._const_names:
            env[name] = self._const_q[name] if mode == "integer" else graph.initializers[name]
        last_use = {}
        for idx, node in enumerate(graph.nodes):
            for n in node.inputs:
                last_use[n] = idx
        keep = set(graph.outputs)
        for idx, node in enumerate(graph.nodes):
            layer = self.quant_layers[node.name]
            ins = [env[n] for n in layer.data_inputs]
            outs = layer.calibrate(ins) if mode == "calibrate" else layer.quantized_infer_integer(ins)
            if trace is not None:
                trace(layer, outs)
            env.update(zip(node.outputs, outs))
            for n in set(layer.data_inputs):
                if last_use.get(n) == idx and n not in keep:
                    env.pop(n, None)
        results = []
        for name in graph.outputs:
            value = env[name]
            if mode == "integer":
                qp = self.qparams[name]
                value = self.lib.dequantize_f32(value, qp.scale, qp.zp)
            results.append(value)
        return results[0] if len(results) == 1 else results

    def compare_layers(self, x, mode="integer"):
        """Per-layer error of the integer pass against the float pass
        (quant_container.py:196-223): ``{layer name: {"max_diff",
        "mean_diff", "layer_type"}}``, each layer's dequantized outputs
        against the float run's on the same input.  The fake-quant mode of
        the reference is not part of this build."""
        if mode != "integer":
            raise ValueError("mode must be 'integer' (fake-quant is not provided)")
        float_env = float_ops.run_float(self.graph, x, keep_all=True, lib=self.lib)
        comparison = {}

        def trace(layer, outs):
            diffs = []
            for name, q in zip(layer.node.outputs, outs):
                qp = self.qparams[name]
                deq = self.lib.dequantize_f32(np.asarray(q), qp.scale, qp.zp)
                diffs.append(np.abs(float_env[name] - deq))
            comparison[layer.name] = {
                "max_diff": float(max(d.max() for d in diffs)),
                "mean_diff": float(np.mean([d.mean() for d in diffs])),
                "layer_type": layer.node.op_type,
            }

        self._execute(x, mode, trace=trace)
        return comparison

    def run_integer_raw(self, x):
        """Integer pass returning the graph outputs as int32 tensors (no
        final dequantize) -- the bit-exact comparison surface."""
        if not self.calibrated:
            raise ValueError("Container is not calibrated; call calibrate().")
        env = self.quantize_inputs(float_ops.normalize_feeds(self.graph, x))
        for name in self._const_names:
            env[name] = self._const_q[name]
        for node in self.graph.nodes:
            layer = self.quant_layers[node.name]
            env.update(zip(node.outputs,
                           layer.quantized_infer_integer([env[n] for n in layer.data_inputs])))
        outs = [env[n] for n in self.graph.outputs]
        return outs[0] if len(outs) == 1 else outs

    # ---------------------------------------------------------- persistence --
    def save(self, path):
        """q.json: quant_type, per_channel and every tensor's qparams
        (quant_container.py:226-237)."""
        payload = {"quant_type": self.quant_type, "per_channel": self.per_channel,
                   "qparams": {k: v.to_dict() for k, v in self.qparams.items()}}
        Path(path).write_text(json.dumps(payload, indent=2))

    @classmethod
    def load(cls, graph, path, lib=None):
        """Rebuilds a calibrated container from the graph and a q.json
        (quant_container.py:239-267)."""
        payload = json.loads(Path(path).read_text())
        return cls.from_qparams(graph, payload, lib=lib)

    @classmethod
    def from_qparams(cls, graph, payload, lib=None):
        c = cls(graph, payload["quant_type"], payload["per_channel"], lib=lib)
        c.qparams = {k: QParams.from_dict(v) for k, v in payload["qparams"].items()}
        missing = [n for n in graph.input_names + c._const_names if n not in c.qparams]
        if missing:
            raise ValueError(f"saved parameters do not match model: {missing}")
        for name in c._const_names:
            qp = c.qparams[name]
            c._const_q[name] = c.lib.quantize_f32(graph.initializers[name].astype(np.float32),
                                                  qp.scale, qp.zp, qp.qmin, qp.qmax)
        for layer in c.layers:
            layer.load_qparams(c)
        c.calibrated = True
        return c
