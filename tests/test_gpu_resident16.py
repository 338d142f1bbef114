"""Device-resident int16 executor (ResidentNet16) vs the reference (B200).

An int16 graph takes the reference's wide route for every Conv / Gemm
(int32 operands, int64 accumulation).  The resident executor computes it as
byte-split tensor-core products combined exactly in int64, so every integer
tensor must equal the reference's bit for bit; the Softmax float fallback
is allowed 1 output LSB like the int8 tests.
"""
import json

import numpy as np
import pytest
import torch

from quantanything_b200 import networks
from quantanything_b200.container import QuantContainer
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu
GRAPHS = GOLDEN / "graphs"
SOFTMAX_LSB = 1


def _net(name, lib, batch):
    from quantanything_b200.resident16 import ResidentNet16

    meta = json.loads((GRAPHS / f"{name}.meta.json").read_text())
    g = getattr(networks, meta["builder"])(**meta["kwargs"])
    qc = QuantContainer.load(g, GRAPHS / f"{name}.qjson", lib=lib)
    return ResidentNet16(qc, batch), qc, meta


def _run(net, x):
    net.forward_device(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    net.check_status()
    return net.out_q.cpu().numpy()


def _integer_pass(qc, x, stop_at="Softmax"):
    """The container's layer-by-layer integer pass (drop-in ABI route,
    itself pinned bit-exactly to the reference) up to the Softmax."""
    env = dict(qc.quantize_inputs({qc.graph.inputs[0].name: x}))
    for node in qc.graph.nodes:
        if node.op_type == stop_at:
            return env, node.inputs[0]
        layer = qc.quant_layers[node.name]
        outs = layer.quantized_infer_integer([env[n] for n in layer.data_inputs])
        env.update(zip(node.outputs, outs))
    raise AssertionError("no Softmax")


def test_yolov8n_int16_batch2_matches_reference(gpu_lib):
    net, qc, meta = _net("yolov8n_cls_int16", gpu_lib, 2)
    assert all(p.desc.groups == 1 for k, p in net.steps if k == "conv")
    x = networks.images(2, 224, seed=meta["eval_seed"])
    q = _run(net, x)
    ref = np.load(GRAPHS / "yolov8n_cls_int16.npz")["q"]
    assert np.abs(q.astype(np.int64) - ref).max() <= SOFTMAX_LSB
    env, logits = _integer_pass(qc, x)
    got = net.tensor(logits).cpu().numpy().reshape(env[logits].shape)
    np.testing.assert_array_equal(got, env[logits])


def test_yolov8n_int16_every_tensor_bit_exact(gpu_lib):
    """Each planned tensor (convolution outputs with their fused LUT / Add,
    Concat buffers, the pooled features) equals the drop-in pass's."""
    net, qc, meta = _net("yolov8n_cls_int16", gpu_lib, 2)
    x = networks.images(2, 224, seed=11)
    _run(net, x)
    env, _ = _integer_pass(qc, x)
    checked = 0
    for name, view in net._views.items():
        if name not in env or name == qc.graph.inputs[0].name:
            continue
        got = net.tensor(name).cpu().numpy().reshape(env[name].shape)
        np.testing.assert_array_equal(got, env[name], err_msg=name)
        checked += 1
    assert checked >= 20


def test_yolo_mini_int16_grouped_and_fused(gpu_lib):
    """The small YOLO graph: depthwise conv on the CUDA-core route, fused
    LUT / residual Add / Concat copies on the tensor-core route."""
    net, qc, meta = _net("yolo_mini_int16", gpu_lib, 2)
    assert any(p.desc.groups > 1 for k, p in net.steps if k == "conv")
    x = networks.images(2, meta["image"], seed=meta["eval_seed"])
    q = _run(net, x)
    ref = np.load(GRAPHS / "yolo_mini_int16.npz")["q"]
    assert np.abs(q.astype(np.int64) - ref).max() <= SOFTMAX_LSB
    env, logits = _integer_pass(qc, x)
    got = net.tensor(logits).cpu().numpy().reshape(env[logits].shape)
    np.testing.assert_array_equal(got, env[logits])


def test_int16_batch_invariance_and_graph_replay(gpu_lib):
    """Images 0..3 of a batch of 8 equal a batch of 4 (batch sharding is
    exact), and CUDA-graph replay equals the eager pass."""
    net8, _, _ = _net("yolov8n_cls_int16", gpu_lib, 8)
    net4, _, _ = _net("yolov8n_cls_int16", gpu_lib, 4)
    x = networks.images(8, 224, seed=5)
    eager = _run(net8, x).copy()
    np.testing.assert_array_equal(eager[:4], _run(net4, x[:4]))
    net8.capture()
    for _ in range(2):
        net8.replay()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(net8.out_q.cpu().numpy(), eager)
    np.testing.assert_array_equal(net8.run(x), net8.out_f32.cpu().numpy())


def test_sppf_mini_int16_maxpool(gpu_lib, oracle, tmp_path):
    """The SPPF block (three chained MaxPool k5 s1 p2, padded with qmin, into
    a Concat) on the int16 executor: calibrated on the C oracle, the same
    q.json loaded for the GPU; the logits equal the oracle's layer-by-layer
    integer pass bit for bit, the Softmax output within 1 LSB."""
    from quantanything_b200.resident16 import ResidentNet16

    g = networks.sppf_mini(width=16)
    qc = QuantContainer(g, "int16", per_channel=True, lib=oracle)
    qc.calibrate([networks.images(4, 32, seed=s) for s in range(2)])
    qc.save(tmp_path / "sppf_mini_int16.qjson")
    net = ResidentNet16(QuantContainer.load(g, tmp_path / "sppf_mini_int16.qjson",
                                            lib=gpu_lib), 2)
    assert sum(kind == "maxpool" for kind, _ in net.steps) == 3
    x = networks.images(2, 32, seed=7)
    q = _run(net, x)
    assert np.abs(q.astype(np.int64) - qc.run_integer_raw(x)).max() <= SOFTMAX_LSB
    env, logits = _integer_pass(qc, x)
    got = net.tensor(logits).cpu().numpy().reshape(env[logits].shape)
    np.testing.assert_array_equal(got, env[logits])


@pytest.mark.parametrize("name", ["yolo_mini_uint8", "sppf_mini_uint8"])
def test_uint8_graphs_on_the_16bit_route(gpu_lib, name):
    """uint8 graphs (asymmetric activations and weights: centred weights up
    to +-255) run on the int16 executor; the reference's golden outputs
    within the Softmax's 1 LSB, the logits equal to the drop-in pass."""
    net, qc, meta = _net(name, gpu_lib, 2)
    x = networks.images(2, meta["image"], seed=meta["eval_seed"])
    q = _run(net, x)
    ref = np.load(GRAPHS / f"{name}.npz")["q"]
    assert np.abs(q.astype(np.int64) - ref).max() <= SOFTMAX_LSB
    env, logits = _integer_pass(qc, x)
    got = net.tensor(logits).cpu().numpy().reshape(env[logits].shape)
    np.testing.assert_array_equal(got, env[logits])


@pytest.mark.parametrize("name", ["yolo_mini_uint16", "sppf_mini_uint16", "shaping_mini_uint16",
                                  "yolov8n_cls_uint16"])
def test_uint16_graphs_match_reference(gpu_lib, name):
    """uint16 graphs on the resident 16-bit route: activations stored 32768
    lower in the signed planes, 17-bit centred weights in three byte planes
    (six 8-bit tensor-core products per K-step).  Every planned tensor must
    equal the drop-in pass's (itself pinned to the reference) and the
    output the reference's within the Softmax fallback's LSB."""
    from quantanything_b200.resident import make_resident
    from quantanything_b200.resident16 import ResidentNet16

    meta = json.loads((GRAPHS / f"{name}.meta.json").read_text())
    g = getattr(networks, meta["builder"])(**meta["kwargs"])
    qc = QuantContainer.load(g, GRAPHS / f"{name}.qjson", lib=gpu_lib)
    net = make_resident(qc, meta["eval_batch"])
    assert isinstance(net, ResidentNet16) and net._w_planes == 3
    x = networks.images(meta["eval_batch"], meta["image"], seed=meta["eval_seed"])
    net.forward_device(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    net.check_status()
    ref = np.load(GRAPHS / f"{name}.npz")
    q = net.output_int().cpu().numpy().astype(np.int64)
    assert q.min() >= 0 and np.abs(q - ref["q"]).max() <= SOFTMAX_LSB
    env, _ = _integer_pass(qc, x)
    # a tensor whose consumers are all Concats lands in the Concat's buffer
    # (rescaled in the producer's epilogue); its own view is never written
    concat_only = {t for t in net._views
                   if all(n.op_type == "Concat" for n in g.nodes if t in n.inputs)
                   and any(t in n.inputs for n in g.nodes)}
    checked = 0
    for tname in net._views:
        if tname not in env or tname == qc.graph.inputs[0].name or tname in concat_only:
            continue
        got = net.tensor(tname).cpu().numpy().reshape(env[tname].shape)
        np.testing.assert_array_equal(got, env[tname], err_msg=tname)
        checked += 1
    assert checked >= 5
