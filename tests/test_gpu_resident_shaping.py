"""Resident Pad / Slice / Transpose vs the reference's integer pass (B200).

The reference's scale-preserving layout operators (quant_layers.py:593-650;
Pad fills with the input zero point) on the reference-generated
``shaping_mini`` fixtures, int8 on ResidentNet and int16 on ResidentNet16:
an aligned channel Slice is a view, every other form a window copy.  Every
tensor the executor keeps must equal the host mirror's bit for bit (the
mirror, on the C oracle, is pinned to the reference), and the graph output
must match the reference's within the Softmax fallback's 1 LSB.
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
SOFTMAX_LSB = 1


def _mirror_env(qc, x):
    env = qc.quantize_inputs(float_ops.normalize_feeds(qc.graph, x))
    for n in qc._const_names:
        env[n] = qc._const_q[n]
    for node in qc.graph.nodes:
        layer = qc.quant_layers[node.name]
        env.update(zip(node.outputs,
                       layer.quantized_infer_integer([env[n] for n in layer.data_inputs])))
    return env


@pytest.mark.parametrize("name", ["shaping_mini_int8", "shaping_mini_int16"])
def test_shaping_graph_matches_reference(gpu_lib, oracle, name):
    from quantanything_b200.resident import make_resident

    meta = json.loads((GRAPHS / f"{name}.meta.json").read_text())
    g = networks.shaping_mini(**meta["kwargs"])
    qc = QuantContainer.load(g, GRAPHS / f"{name}.qjson", lib=gpu_lib)
    net = make_resident(qc, meta["eval_batch"])
    kinds = [k for k, _ in net.steps]
    assert kinds.count("window") == 6  # two Pads, two Transposes, two of three Slices
    x = networks.images(meta["eval_batch"], meta["image"], seed=meta["eval_seed"])
    net.forward_device(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    net.check_status()
    env = _mirror_env(QuantContainer.load(g, GRAPHS / f"{name}.qjson", lib=oracle), x)
    checked = 0
    for tname in net._views:
        if tname == g.inputs[0].name or tname not in env:
            continue
        got = net.tensor(tname).cpu().numpy().reshape(-1)
        np.testing.assert_array_equal(got, np.asarray(env[tname]).reshape(-1), err_msg=tname)
        checked += 1
    assert checked >= 12
    ref = np.load(GRAPHS / f"{name}.npz")["q"].astype(np.int64)
    q = net.output_int().cpu().numpy().astype(np.int64)
    assert np.abs(q - ref).max() <= SOFTMAX_LSB
