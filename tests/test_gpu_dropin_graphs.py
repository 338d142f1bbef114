"""Drop-in route on the GPU: whole quantized graphs, layer by layer.

The container drives the CUDA library's host-pointer ABI exactly as the
reference's QuantContainer drives its C++ library under QA_LIB (one kernel
call per layer on host int32 tensors).  Every network's int32 output must
equal the reference's bit for bit -- including the int16 YOLOv8n-cls
(configuration 4: every contraction on the wide int64 route) and the
uint8 graphs (asymmetric zero points).
"""
import json

import numpy as np
import pytest

from quantanything_b200 import networks
from quantanything_b200.container import QuantContainer
from tests.conftest import GOLDEN
from tests.golden.graph_fixtures import NETWORKS

pytestmark = pytest.mark.gpu
GRAPHS = GOLDEN / "graphs"


@pytest.mark.parametrize("name", sorted(NETWORKS))
def test_dropin_graph_matches_reference(gpu_lib, name):
    meta = json.loads((GRAPHS / f"{name}.meta.json").read_text())
    g = getattr(networks, meta["builder"])(**meta["kwargs"])
    qc = QuantContainer.load(g, GRAPHS / f"{name}.qjson", lib=gpu_lib)
    x = networks.images(meta["eval_batch"], meta["image"], seed=meta["eval_seed"])
    ref = np.load(GRAPHS / f"{name}.npz")
    np.testing.assert_array_equal(qc.run_integer_raw(x), ref["q"])
    y = qc.run_graph(x, "integer")
    np.testing.assert_array_equal(y.view(np.uint32), ref["y"].view(np.uint32))
