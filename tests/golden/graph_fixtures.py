"""Graph-level golden fixtures produced by the reference's QuantContainer.

Called by make_golden.py (--graphs) with the reference importable.  For each
network below the REFERENCE calibrates on seeded images, writes its q.json,
and runs its integer pass on a seeded batch; we store the q.json, the int32
graph output, its dequantized float32 form, and SHA-256 digests of every
layer's prepared integer parameters.  The networks are this package's
seeded builders (quantanything_b200.networks), converted node by node into
the reference's own OnnxGraph/Node classes.
"""
import json

import numpy as np

from tests.golden.make_golden import digest

NETWORKS = {
    # name: (builder, kwargs, quant_type, calib batches, calib batch size, eval batch)
    "yolo_mini_int8": ("yolo_mini", {"width": 16}, "int8", 2, 4, 2),
    "yolo_mini_uint8": ("yolo_mini", {"width": 16}, "uint8", 2, 4, 2),
    "yolo_mini_int16": ("yolo_mini", {"width": 16}, "int16", 2, 4, 2),
    "yolov8n_cls_int8": ("yolov8n_cls", {}, "int8", 4, 8, 2),
    "yolov8n_cls_int16": ("yolov8n_cls", {}, "int16", 4, 8, 2),
    "sppf_mini_int8": ("sppf_mini", {"width": 16}, "int8", 2, 4, 2),
    "sppf_mini_uint8": ("sppf_mini", {"width": 16}, "uint8", 2, 4, 2),
    "shaping_mini_int8": ("shaping_mini", {"width": 16}, "int8", 2, 4, 2),
    "shaping_mini_int16": ("shaping_mini", {"width": 16}, "int16", 2, 4, 2),
    # uint16: asymmetric 16-bit activations and weights (17-bit centred weights)
    "yolo_mini_uint16": ("yolo_mini", {"width": 16}, "uint16", 2, 4, 2),
    "sppf_mini_uint16": ("sppf_mini", {"width": 16}, "uint16", 2, 4, 2),
    "shaping_mini_uint16": ("shaping_mini", {"width": 16}, "uint16", 2, 4, 2),
    "yolov8n_cls_uint16": ("yolov8n_cls", {}, "uint16", 4, 8, 2),
    # the batch is static in a ViT graph: calibration and evaluation use it
    "vit_mini_int8": ("vit", {"batch": 4}, "int8", 2, 4, 4),
    "vit_mini_int16": ("vit", {"batch": 4}, "int16", 2, 4, 4),
    "vit_mini_uint16": ("vit", {"batch": 4}, "uint16", 2, 4, 4),
    # stand-alone activation x activation MatMuls (no head split, no Softmax)
    "vit_gram_mini_int8": ("vit", {"batch": 4, "attention": "gram"}, "int8", 2, 4, 4),
    # ViT-B/16 (cfg3's model) at batch 2: the full-size parity case
    "vit_b16_int8": ("vit", {"img": 224, "patch": 16, "dim": 768, "heads": 12, "depth": 12,
                             "classes": 1000, "batch": 2, "std": 0.02}, "int8", 2, 2, 2),
}


def to_reference_graph(g):
    from quantization.onnx_graph import Node as RNode
    from quantization.onnx_graph import OnnxGraph, ValueInfo as RVI

    def conv(n):
        attrs = dict(n.attrs)
        if n.op_type == "FusedElementwise":
            attrs["nodes"] = [conv(s) for s in n.attrs["nodes"]]
        return RNode(n.name, n.op_type, list(n.inputs), list(n.outputs), attrs)

    inputs = [RVI(v.name, v.shape, np.float32) for v in g.inputs]
    return OnnxGraph([conv(n) for n in g.nodes], dict(g.initializers), inputs, list(g.outputs),
                     g.opset)


def layer_digests(container):
    out = {}
    for layer in container.layers:
        d = {"type": type(layer).__name__}
        for attr in ("w_centered", "bias_int", "q_mult", "shift", "lut", "q_B"):
            v = getattr(layer, attr, None)
            if v is not None:
                d[attr] = digest(np.asarray(v))
        for attr in ("lut_offset", "wide"):
            if hasattr(layer, attr):
                d[attr] = int(getattr(layer, attr))
        if hasattr(layer, "_mult"):
            d["mult"] = [list(map(int, m)) for m in layer._mult] if isinstance(
                layer._mult, list) else int(layer._mult)
        out[layer.name] = d
    return out


def generate(outdir, only=None):
    from quantanything_b200 import networks
    from quantization import QuantContainer

    outdir.mkdir(parents=True, exist_ok=True)
    for name, (builder, kw, qtype, nb, bs, ne) in NETWORKS.items():
        if only and name not in only:
            continue
        g = getattr(networks, builder)(**kw)
        size = g.inputs[0].shape[2]
        rg = to_reference_graph(g)
        qc = QuantContainer(rg, quant_type=qtype, per_channel=True)
        calib = [networks.images(bs, size, seed=100 + i) for i in range(nb)]
        qc.calibrate(calib)
        qc.save(outdir / f"{name}.qjson")
        x = networks.images(ne, size, seed=7)
        env, out = qc._execute(x, "integer")
        q = env[rg.outputs[0]]
        # inputs are not stored: networks.images(ne, size, seed=7) regenerates them
        extra = {}
        if name == "yolov8n_cls_int8":
            # the benchmark batch: 64 images, pinned by digest
            x64 = networks.images(64, size, seed=7)
            env64, _ = qc._execute(x64, "integer", trace=lambda layer, outs: None)
            extra["q64_digest"] = digest(np.asarray(env64[rg.outputs[0]], np.int32))
            gemm = [n for n in rg.nodes if n.op_type == "Gemm"][0]
            extra["logits64_digest"] = digest(np.asarray(env64[gemm.outputs[0]], np.int32))
            extra["logits_name"] = gemm.outputs[0]
            np.save(outdir / "yolov8n_cls_int8.q64.npy", np.asarray(env64[rg.outputs[0]],
                                                                   np.int8))
        np.savez_compressed(outdir / f"{name}.npz", q=np.asarray(q, np.int32),
                            y=np.asarray(out, np.float32))
        meta = {"builder": builder, "kwargs": kw, "quant_type": qtype, "eval_batch": ne,
                "eval_seed": 7, "image": size, **extra}
        (outdir / f"{name}.meta.json").write_text(json.dumps(meta, indent=1))
        (outdir / f"{name}.layers.json").write_text(json.dumps(layer_digests(qc), indent=1))
        print("graph fixture", name, q.shape)
