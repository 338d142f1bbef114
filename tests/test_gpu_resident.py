"""Device-resident fused executor vs the reference's integer pass (B200).

The container is loaded from the reference's own q.json; every integer
tensor must match the reference bit for bit.  The Softmax float fallback is
allowed 1 output LSB (the tolerance the task states for float fallbacks):
float64 exp / summation order on the GPU may differ from NumPy's in the
last ulp.
"""
import json

import numpy as np
import pytest
import torch

from quantanything_b200 import networks
from quantanything_b200.container import QuantContainer
from tests.conftest import GOLDEN
from tests.test_oracle_golden import _digest

pytestmark = pytest.mark.gpu
GRAPHS = GOLDEN / "graphs"
SOFTMAX_LSB = 1


def _net(name, lib, batch, **kw):
    from quantanything_b200.resident import ResidentNet

    meta = json.loads((GRAPHS / f"{name}.meta.json").read_text())
    g = getattr(networks, meta["builder"])(**meta["kwargs"])
    qc = QuantContainer.load(g, GRAPHS / f"{name}.qjson", lib=lib)
    return ResidentNet(qc, batch, **kw), qc, meta


def _run(net, x):
    net.forward_device(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    net.check_status()
    return net.out_q.cpu().numpy()


def test_yolov8n_int8_batch2_matches_reference(gpu_lib):
    net, qc, meta = _net("yolov8n_cls_int8", gpu_lib, 2)
    x = networks.images(2, 224, seed=meta["eval_seed"])
    q = _run(net, x)
    ref = np.load(GRAPHS / "yolov8n_cls_int8.npz")["q"]
    assert np.abs(q.astype(np.int64) - ref).max() <= SOFTMAX_LSB
    assert (q == ref).mean() > 0.999
    # every integer tensor before the Softmax, against the drop-in ABI pass
    # of the same container (itself pinned to the reference)
    env = {}
    feeds = qc.quantize_inputs({"images": x})
    env.update(feeds)
    for node in qc.graph.nodes:
        layer = qc.quant_layers[node.name]
        if node.op_type == "Softmax":
            break
        outs = layer.quantized_infer_integer([env[n] for n in layer.data_inputs])
        env.update(zip(node.outputs, outs))
    logits = meta["logits_name"]
    got = net.tensor(logits).cpu().numpy().reshape(env[logits].shape)
    np.testing.assert_array_equal(got, env[logits])


def test_yolov8n_int8_batch64_logits_digest(gpu_lib):
    """The benchmark batch: 64 images, logits bit-exact (digest of the
    reference's int32 Gemm output), Softmax within 1 LSB."""
    net, qc, meta = _net("yolov8n_cls_int8", gpu_lib, 64)
    x = networks.images(64, 224, seed=meta["eval_seed"])
    q = _run(net, x)
    logits = net.tensor(meta["logits_name"]).cpu().numpy().reshape(64, -1)
    assert _digest(logits.astype(np.int32)) == meta["logits64_digest"]
    ref = np.load(GRAPHS / "yolov8n_cls_int8.q64.npy").astype(np.int64)
    assert np.abs(q.astype(np.int64) - ref).max() <= SOFTMAX_LSB


def test_cuda_graph_replay_matches_eager(gpu_lib):
    net, qc, meta = _net("yolov8n_cls_int8", gpu_lib, 8)
    x = networks.images(8, 224, seed=3)
    eager = _run(net, x).copy()
    net.capture()
    for _ in range(3):
        net.replay()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(net.out_q.cpu().numpy(), eager)
    host = net.run(x)
    np.testing.assert_array_equal(host, net.out_f32.cpu().numpy())


def test_yolo_mini_int8_grouped_and_fused(gpu_lib):
    net, qc, meta = _net("yolo_mini_int8", gpu_lib, 2)
    x = networks.images(2, meta["image"], seed=meta["eval_seed"])
    q = _run(net, x)
    ref = np.load(GRAPHS / "yolo_mini_int8.npz")["q"]
    assert np.abs(q.astype(np.int64) - ref).max() <= SOFTMAX_LSB


@pytest.mark.parametrize("name,batch", [("yolov8n_cls_int8", 3), ("yolo_mini_int8", 2)])
def test_fused_input_layer_matches_separate_path(gpu_lib, name, batch):
    """qa_conv_input_fused_dev (quantize + stem conv in one kernel) gives the
    same integer tensors as the quantize kernel + tensor-core conv."""
    fused, _, meta = _net(name, gpu_lib, batch, fuse_input=True)
    plain, _, _ = _net(name, gpu_lib, batch, fuse_input=False)
    assert fused.steps[0][0] == "conv_input" and plain.steps[0][0] == "quantize"
    x = networks.images(batch, meta["image"], seed=21)
    np.testing.assert_array_equal(_run(fused, x), _run(plain, x))


def test_fused_input_layer_special_values(gpu_lib):
    """The fused input layer on images full of hard cases for its float
    quantizer -- products near rounding ties (a few ulps either side of
    (k + 1/2) * scale), NaN, +-inf, values far beyond the clamp range --
    gives every integer tensor of the separate quantize kernel + conv path
    (itself pinned to the oracle's qa_quantize_f32 / conv)."""
    fused, qc, meta = _net("yolov8n_cls_int8", gpu_lib, 2, fuse_input=True)
    plain, _, _ = _net("yolov8n_cls_int8", gpu_lib, 2, fuse_input=False)
    qp = qc.qparams[qc.graph.inputs[0].name]
    rng = np.random.default_rng(77)
    x = networks.images(2, 224, seed=5)
    flat = x.reshape(-1)
    k = rng.integers(qp.qmin - qp.zp - 2, qp.qmax - qp.zp + 2, flat.size)
    ties = ((k + 0.5) * qp.scale).astype(np.float32)
    ulps = rng.integers(-3, 4, flat.size).astype(np.int32)
    near = (ties.view(np.int32) + ulps).view(np.float32)
    pick = rng.random(flat.size)
    flat[pick < 0.3] = near[pick < 0.3]
    flat[(pick >= 0.3) & (pick < 0.301)] = np.nan
    flat[(pick >= 0.301) & (pick < 0.302)] = np.inf
    flat[(pick >= 0.302) & (pick < 0.303)] = -np.inf
    flat[(pick >= 0.303) & (pick < 0.31)] *= 1e6
    _run(fused, x)
    _run(plain, x)
    names = [n for n in fused._views if n in plain._views and n != qc.graph.inputs[0].name]
    assert names
    for n in names:
        np.testing.assert_array_equal(fused.tensor(n).cpu().numpy(), plain.tensor(n).cpu().numpy(),
                                      err_msg=n)


def test_sppf_mini_int8_maxpool(gpu_lib):
    """Resident MaxPool (padded with qmin) chained three times into a Concat."""
    net, qc, meta = _net("sppf_mini_int8", gpu_lib, 2)
    assert any(kind == "maxpool" for kind, _ in net.steps)
    x = networks.images(2, meta["image"], seed=meta["eval_seed"])
    q = _run(net, x)
    ref = np.load(GRAPHS / "sppf_mini_int8.npz")["q"]
    assert np.abs(q.astype(np.int64) - ref).max() <= SOFTMAX_LSB


def test_batch_invariance(gpu_lib):
    """Batch sharding is exact: images 0..3 of a batch of 8 equal a batch of 4
    (the reference's batch-size invariance, test_container.py:201-206)."""
    net8, _, _ = _net("yolov8n_cls_int8", gpu_lib, 8)
    net4, _, _ = _net("yolov8n_cls_int8", gpu_lib, 4)
    x = networks.images(8, 224, seed=5)
    np.testing.assert_array_equal(_run(net8, x)[:4], _run(net4, x[:4]))


def test_wide_weights_are_rejected_cleanly(gpu_lib):
    from quantanything_b200.resident import UnsupportedGraph

    with pytest.raises(UnsupportedGraph):
        _net("yolo_mini_int16", gpu_lib, 2)


def test_pipelined_host_calls_match_single_runs(gpu_lib):
    """run_pipelined (copies of batch i+1 overlapped with the forward of
    batch i through two staging buffers) returns, per batch, exactly what
    run() returns for that batch alone."""
    net, _, _ = _net("yolov8n_cls_int8", gpu_lib, 4)
    xs = [networks.images(4, 224, seed=40 + i) for i in range(5)]
    want = [net.run(x).copy() for x in xs]
    xs_pinned = [torch.from_numpy(x).pin_memory() for x in xs]
    outs = [torch.empty((4, 1000), dtype=torch.float32).pin_memory() for _ in xs]
    net.run_pipelined(xs_pinned, outs)
    torch.cuda.current_stream().synchronize()
    for w, o in zip(want, outs):
        np.testing.assert_array_equal(o.numpy(), w)


def test_traced_forward_matches_plain(gpu_lib):
    """forward_traced (NVTX range per launch) computes the same outputs."""
    net, _, _ = _net("yolo_mini_int8", gpu_lib, 2)
    x = networks.images(2, 32, seed=3)
    plain = _run(net, x).copy()
    net.forward_traced(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(net.out_q.cpu().numpy(), plain)


@pytest.mark.parametrize("name,cls", [("yolo_mini_int8", "ResidentNet"),
                                      ("yolo_mini_uint8", "ResidentNet16"),
                                      ("yolo_mini_int16", "ResidentNet16"),
                                      ("vit_mini_int8", "ResidentViT")])
def test_make_resident_picks_the_executor(gpu_lib, name, cls):
    from quantanything_b200.resident import make_resident

    meta = json.loads((GRAPHS / f"{name}.meta.json").read_text())
    g = getattr(networks, meta["builder"])(**meta["kwargs"])
    qc = QuantContainer.load(g, GRAPHS / f"{name}.qjson", lib=gpu_lib)
    net = make_resident(qc, meta["eval_batch"])
    assert type(net).__name__ == cls
    x = networks.images(meta["eval_batch"], meta["image"], seed=meta["eval_seed"])
    q = _run(net, x)
    ref = np.load(GRAPHS / f"{name}.npz")["q"]
    assert np.abs(q.astype(np.int64) - ref).max() <= SOFTMAX_LSB


@pytest.mark.parametrize("name,batch", [("yolov8n_cls_int8", 64), ("yolov8n_cls_int8", 33)])
def test_gap_fused_into_head_conv_matches_separate_pool(gpu_lib, name, batch):
    """GlobalAveragePool folded into the head conv's epilogue (per-image
    channel sums, the completing warp requantizes) equals the separate
    pooling kernel bit for bit, with one launch less, on every tensor;
    repeated forwards (CUDA-graph replays) leave the sums clean."""
    fused, qc, meta = _net(name, gpu_lib, batch)
    plain, _, _ = _net(name, gpu_lib, batch, fuse_gap=False)
    kinds_f = [k for k, _ in fused.steps]
    kinds_p = [k for k, _ in plain.steps]
    assert "gap" not in kinds_f and "gap" in kinds_p and len(kinds_f) == len(kinds_p) - 1
    assert any(getattr(p, "gap", None) is not None for k, p in fused.steps if k == "conv")
    for seed in (3, 4):
        x = networks.images(batch, meta["image"], seed=seed)
        qf = _run(fused, x)
        qp = _run(plain, x)
        np.testing.assert_array_equal(qf, qp)
        for n in fused._views:
            if n == qc.graph.inputs[0].name:
                continue
            np.testing.assert_array_equal(fused.tensor(n).cpu().numpy(),
                                          plain.tensor(n).cpu().numpy(), err_msg=n)
    fused.capture()
    for _ in range(3):
        fused.replay()
    torch.cuda.synchronize()
    fused.check_status()
    np.testing.assert_array_equal(fused.out_q.cpu().numpy(), qp)
