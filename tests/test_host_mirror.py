"""The host mirror (layers / container) reproduces the reference exactly.

Runs on the CPU with the C oracle as the kernel library: loading the
reference's q.json must re-derive every layer's integer parameters with the
same digests the reference produced, and the drop-in integer pass must give
the reference's int32 outputs bit for bit.
"""
import json

import numpy as np
import pytest

from quantanything_b200 import networks
from quantanything_b200.container import QuantContainer
from tests.conftest import GOLDEN
from tests.golden.graph_fixtures import NETWORKS, layer_digests

GRAPHS = GOLDEN / "graphs"


def load(name, lib):
    meta = json.loads((GRAPHS / f"{name}.meta.json").read_text())
    g = getattr(networks, meta["builder"])(**meta["kwargs"])
    qc = QuantContainer.load(g, GRAPHS / f"{name}.qjson", lib=lib)
    return qc, meta


@pytest.mark.parametrize("name", sorted(NETWORKS))
def test_prepared_parameters_match_reference(oracle, name):
    qc, _ = load(name, oracle)
    ref = json.loads((GRAPHS / f"{name}.layers.json").read_text())
    got = layer_digests(qc)
    assert list(got) == list(ref)
    for lname in ref:
        assert got[lname] == ref[lname], lname


@pytest.mark.parametrize("name", ["yolo_mini_int8", "yolo_mini_uint8", "yolo_mini_int16",
                                  "yolov8n_cls_int8", "sppf_mini_int8", "sppf_mini_uint8",
                                  "vit_mini_int8", "vit_mini_int16", "yolo_mini_uint16",
                                  "sppf_mini_uint16", "shaping_mini_uint16", "vit_mini_uint16"])
def test_integer_outputs_match_reference(oracle, name):
    qc, meta = load(name, oracle)
    x = networks.images(meta["eval_batch"], meta["image"], seed=meta["eval_seed"])
    ref = np.load(GRAPHS / f"{name}.npz")
    q = qc.run_integer_raw(x)
    np.testing.assert_array_equal(q, ref["q"])
    y = qc.run_graph(x, "integer")
    np.testing.assert_array_equal(y.view(np.uint32), ref["y"].view(np.uint32))


def test_qjson_roundtrip(oracle, tmp_path):
    qc, _ = load("yolo_mini_int8", oracle)
    qc.save(tmp_path / "q.json")
    again = json.loads((tmp_path / "q.json").read_text())
    assert again == json.loads((GRAPHS / "yolo_mini_int8.qjson").read_text())


def test_load_rejects_mismatched_qparams(oracle, tmp_path):
    payload = json.loads((GRAPHS / "yolo_mini_int8.qjson").read_text())
    del payload["qparams"]["images"]
    (tmp_path / "bad.json").write_text(json.dumps(payload))
    with pytest.raises(ValueError):
        QuantContainer.load(networks.yolo_mini(width=16), tmp_path / "bad.json", lib=oracle)


def test_compare_layers_reports_every_layer(oracle):
    """compare_layers (quant_container.py:196-223): one entry per layer, the
    integer pass tracking the float pass (small errors on an int8 graph)."""
    from quantanything_b200 import networks
    from quantanything_b200.container import QuantContainer

    g = networks.yolo_mini(width=16)
    qc = QuantContainer.load(g, GRAPHS / "yolo_mini_int8.qjson", lib=oracle)
    cmp = qc.compare_layers(networks.images(2, 32, seed=7))
    assert set(cmp) == {layer.name for layer in qc.layers}
    assert all(v["max_diff"] >= v["mean_diff"] >= 0 for v in cmp.values())
    first_conv = next(k for k, v in cmp.items() if v["layer_type"] == "Conv")
    assert cmp[first_conv]["mean_diff"] < 0.05
