"""The reference's unchanged Python on top of the CUDA library (B200).

With QA_LIB pointing at libqa_kernels.so, the reference's own
QuantContainer and quant_layers (its installed package, baseline/_ref)
run the integer pass of every golden fixture -- int8, uint8 and int16
YOLO-style graphs, SPPF, the int8 / int16 ViT minis and YOLOv8n-cls --
with each layer's kernels executed by the CUDA library through the
reference's ctypes loader.  The int32 outputs and the dequantized float32
outputs must equal the reference-generated fixtures bit for bit, and the
reference's native.* wrappers must return exact results.  Skipped when the
reference package is not installed.
"""
import json
import subprocess
import sys

import pytest

from tests.conftest import REPO
from tests.reference_dropin import GRAPH_CASES, reference_package_dir

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(reference_package_dir() is None,
                                 reason="reference package not installed")]


def test_reference_container_runs_on_the_cuda_library(gpu_lib):
    proc = subprocess.run([sys.executable, str(REPO / "tests" / "reference_dropin.py"),
                           "graphs", str(gpu_lib.path)], capture_output=True, text=True,
                          timeout=900)
    assert proc.returncode == 0, proc.stderr[-3000:]
    res = json.loads(proc.stdout.strip().splitlines()[-1])
    assert sorted(res["graphs"]) == sorted(GRAPH_CASES)
    for name, r in res["graphs"].items():
        assert r["int_equal"] and r["float_equal"], (name, r)
    assert res["kernels"] and all(res["kernels"].values()), res["kernels"]
