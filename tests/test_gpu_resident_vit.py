"""Device-resident ViT (B200) vs the reference's integer pass.

The reference's q.json drives both; every tensor the executor keeps on the
device is compared with the host mirror's tensor of the same name (the
mirror itself is pinned to the reference's output).  Integer layers must
match bit for bit; the float fallbacks (LayerNorm, the attention core) may
differ by one output step on a rounding boundary (their float sums run in
another order than NumPy's), the tolerance stated for float fallbacks.
"""
import json

import numpy as np
import pytest
import torch

from quantanything_b200 import float_ops, networks
from quantanything_b200.container import QuantContainer
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu
GRAPHS = GOLDEN / "graphs"
FALLBACK_LSB = 1
INT16_E2E_LSB = 64  # one-step flips of the float fallbacks, grown through two blocks


def _load(name, lib):
    meta = json.loads((GRAPHS / f"{name}.meta.json").read_text())
    g = networks.vit(**meta["kwargs"])
    return QuantContainer.load(g, GRAPHS / f"{name}.qjson", lib=lib), meta


def _mirror_env(qc, x):
    g = qc.graph
    env = qc.quantize_inputs(float_ops.normalize_feeds(g, x))
    for n in qc._const_names:
        env[n] = qc._const_q[n]
    for node in g.nodes:
        layer = qc.quant_layers[node.name]
        env.update(zip(node.outputs,
                       layer.quantized_infer_integer([env[n] for n in layer.data_inputs])))
    return env


def _run(net, x):
    net.forward_device(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    net.check_status()


def test_vit_mini_int8_matches_reference(gpu_lib):
    from quantanything_b200.resident_vit import ResidentViT

    qc, meta = _load("vit_mini_int8", gpu_lib)
    x = networks.images(meta["eval_batch"], meta["image"], seed=meta["eval_seed"])
    net = ResidentViT(qc, meta["eval_batch"])
    kinds = [k for k, _ in net.steps]
    assert kinds.count("attention") == 2 and kinds.count("layernorm") == 5
    _run(net, x)
    env = _mirror_env(qc, x)
    fallback = {n.outputs[0] for n in qc.graph.nodes
                if n.op_type in ("LayerNormalization", "Reshape")}
    for name in net._views:
        if name == qc.graph.inputs[0].name or name not in env:
            continue
        got = net.tensor(name).cpu().numpy().reshape(-1).astype(np.int64)
        want = np.asarray(env[name]).reshape(-1).astype(np.int64)
        tol = FALLBACK_LSB if name in fallback else 0
        assert np.abs(got - want).max() <= tol, name
    ref = np.load(GRAPHS / "vit_mini_int8.npz")
    q = net.output_int().cpu().numpy()
    # pinned: with these inputs no fallback value lands on a rounding boundary
    np.testing.assert_array_equal(q, ref["q"])
    np.testing.assert_array_equal(net.out_f32.cpu().numpy().view(np.uint32),
                                  ref["y"].view(np.uint32))


def test_vit_graph_replay_matches_eager(gpu_lib):
    from quantanything_b200.resident_vit import ResidentViT

    qc, meta = _load("vit_mini_int8", gpu_lib)
    net = ResidentViT(qc, meta["eval_batch"])
    x = networks.images(meta["eval_batch"], meta["image"], seed=3)
    _run(net, x)
    eager = net.output_int().clone()
    net.capture()
    net.replay()
    torch.cuda.synchronize()
    assert torch.equal(eager, net.output_int())


def test_vit_batch_must_match_the_graph(gpu_lib):
    from quantanything_b200.resident import UnsupportedGraph
    from quantanything_b200.resident_vit import ResidentViT

    qc, meta = _load("vit_mini_int8", gpu_lib)
    with pytest.raises(UnsupportedGraph):
        ResidentViT(qc, meta["eval_batch"] + 1)


def test_vit_mini_int16_resident_against_the_reference(gpu_lib, oracle):
    """int16 ViT on the resident route (ResidentViT16: byte-split tensor-core
    contractions, 16-bit plane kernels for the embedding, LayerNorm, the
    attention core and the Gather).  Each step fed the mirror's inputs:
    integer steps bit-exact, the float fallbacks within one int16 output
    step; end to end the logits stay within INT16_E2E_LSB of the reference's
    and keep its class on every image."""
    from quantanything_b200.resident import make_resident
    from quantanything_b200.resident_vit import ResidentViT16
    from tests.resident_steps import mirror_env, teacher_forced

    qc, meta = _load("vit_mini_int16", gpu_lib)
    net = make_resident(qc, meta["eval_batch"])
    assert isinstance(net, ResidentViT16)
    kinds = [k for k, _ in net.steps]
    assert kinds.count("attention") == 2 and kinds.count("layernorm") == 5
    x = networks.images(meta["eval_batch"], meta["image"], seed=meta["eval_seed"])
    g = qc.graph
    env = mirror_env(QuantContainer.load(g, GRAPHS / "vit_mini_int16.qjson", lib=oracle), x)
    seen = set()
    for i, kind, tname, diff in teacher_forced(net, env, x, g.inputs[0].name):
        seen.add(kind)
        tol = FALLBACK_LSB if kind in ("attention", "layernorm") else 0
        assert diff.max() <= tol, (i, kind, tname, int(diff.max()))
    assert {"conv", "vit_embed", "layernorm", "attention", "gather"} <= seen
    net.forward_device(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    net.check_status()
    ref = np.load(GRAPHS / "vit_mini_int16.npz")["q"].astype(np.int64)
    q = net.output_int().cpu().numpy().astype(np.int64)
    np.testing.assert_array_equal(q.argmax(1), ref.argmax(1))
    assert np.abs(q - ref).max() <= INT16_E2E_LSB


def test_vit_mini_uint16_resident_against_the_reference(gpu_lib, oracle):
    """uint16 ViT on ResidentViT16: activations held 32768 lower in the
    signed planes (every activation zero point, range and table shifted with
    them), 17-bit centred weights in three byte planes.  Teacher-forced
    steps as for int16: integer steps bit-exact, the float fallbacks within
    one output step; end to end the logits stay within INT16_E2E_LSB of the
    reference's and keep its class on every image."""
    from quantanything_b200.resident import make_resident
    from quantanything_b200.resident_vit import ResidentViT16
    from tests.resident_steps import mirror_env, teacher_forced

    qc, meta = _load("vit_mini_uint16", gpu_lib)
    net = make_resident(qc, meta["eval_batch"])
    assert isinstance(net, ResidentViT16) and net._w_planes == 3 and net._act_shift == 32768
    x = networks.images(meta["eval_batch"], meta["image"], seed=meta["eval_seed"])
    g = qc.graph
    env = mirror_env(QuantContainer.load(g, GRAPHS / "vit_mini_uint16.qjson", lib=oracle), x)
    seen = set()
    for i, kind, tname, diff in teacher_forced(net, env, x, g.inputs[0].name):
        seen.add(kind)
        tol = FALLBACK_LSB if kind in ("attention", "layernorm") else 0
        assert diff.max() <= tol, (i, kind, tname, int(diff.max()))
    assert {"conv", "vit_embed", "layernorm", "attention", "gather"} <= seen
    net.forward_device(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    net.check_status()
    ref = np.load(GRAPHS / "vit_mini_uint16.npz")["q"].astype(np.int64)
    q = net.output_int().cpu().numpy().astype(np.int64)
    assert q.min() >= 0
    np.testing.assert_array_equal(q.argmax(1), ref.argmax(1))
    assert np.abs(q - ref).max() <= INT16_E2E_LSB


def test_vit_gram_act_x_act_matmuls_against_the_reference(gpu_lib, oracle):
    """Stand-alone activation x activation MatMuls (the reference's float
    fallback, float_ops.py MatMul, quant_layers.py:195-205) on the resident
    route: qa_matmul_act_bytes_dev reads a [0, 2, 1]-transposed operand in
    place.  Each step fed the mirror's inputs: integer steps bit-exact, the
    MatMuls and LayerNorms within one output step; the logits then keep the
    reference's class."""
    from quantanything_b200.resident_vit import ResidentViT
    from tests.resident_steps import mirror_env, teacher_forced

    name = "vit_gram_mini_int8"
    meta = json.loads((GRAPHS / f"{name}.meta.json").read_text())
    g = networks.vit(**meta["kwargs"])
    qc = QuantContainer.load(g, GRAPHS / f"{name}.qjson", lib=gpu_lib)
    net = ResidentViT(qc, meta["eval_batch"])
    kinds = [k for k, _ in net.steps]
    assert kinds.count("matmul_act") == 2 * meta["kwargs"].get("depth", 2)
    x = networks.images(meta["eval_batch"], meta["image"], seed=meta["eval_seed"])
    env = mirror_env(QuantContainer.load(g, GRAPHS / f"{name}.qjson", lib=oracle), x)
    seen = set()
    for i, kind, tname, diff in teacher_forced(net, env, x, g.inputs[0].name):
        seen.add(kind)
        tol = FALLBACK_LSB if kind in ("matmul_act", "layernorm") else 0
        assert diff.max() <= tol, (i, kind, tname, int(diff.max()))
    assert "matmul_act" in seen
    net.forward_device(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    net.check_status()
    ref = np.load(GRAPHS / f"{name}.npz")["q"]
    np.testing.assert_array_equal(net.output_int().cpu().numpy().argmax(1), ref.argmax(1))
