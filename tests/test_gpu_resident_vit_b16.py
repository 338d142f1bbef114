"""Device-resident ViT-B/16 (configuration 3, the benched transformer) vs the
reference's integer pass, layer by layer and end to end (B200).

Graph, q.json and images are the reference-generated fixture
``vit_b16_int8`` (batch 2, seed 7).  The host mirror of the reference's
integer pass (``quantized_infer_integer`` of every layer,
quant_layers.py:195-205, driven by the reference's own C++ kernels from
oracle/_ref when present, else the C oracle) gives every tensor.

Layer by layer, each resident step is fed the mirror's tensors for its
inputs (teacher forcing) and its outputs are compared with the mirror's:

* integer steps (patch-embedding GEMM, the fused QKV / projection / MLP
  MatMuls with their GELU table and residual Add, the class-token embed,
  the class-token Gather, the head Gemm) must be bit-exact;
* the float fallbacks -- LayerNorm (float_ops.py:336-347) and the attention
  core (scores MatMul, scale Mul, Softmax float_ops.py:380-385, MatMul with
  V float_ops.py:181-186) -- must be within 1 int8 LSB, and on at most
  FALLBACK_FLIP_FRACTION of a step's elements.

End to end, the flips of the float fallbacks propagate through twelve
blocks: the resident logits must keep the reference's class on every image,
stay within E2E_MAX_LSB of the reference's int8 logits, and be bit-identical
on at least E2E_MIN_IDENTICAL of them.
"""
import json
import os

import numpy as np
import pytest
import torch

from quantanything_b200 import networks
from quantanything_b200.container import QuantContainer
from tests.conftest import GOLDEN, REF_LIB, _ensure_oracle
from tests.resident_steps import mirror_env, teacher_forced

pytestmark = pytest.mark.gpu
GRAPHS = GOLDEN / "graphs"
NAME = "vit_b16_int8"
INTEGER_KINDS = ("conv", "vit_embed", "gather")
FALLBACK_KINDS = ("layernorm", "attention")
FALLBACK_LSB = 1
FALLBACK_FLIP_FRACTION = 1e-4
E2E_MAX_LSB = 8
E2E_MIN_IDENTICAL = 0.15


def _mirror_lib():
    from quantanything_b200.native import KernelLibrary

    return KernelLibrary(REF_LIB if REF_LIB.exists() else _ensure_oracle())


@pytest.fixture(scope="module")
def vit_b16(gpu_lib):
    meta = json.loads((GRAPHS / f"{NAME}.meta.json").read_text())
    g = networks.vit(**meta["kwargs"])
    x = networks.images(meta["eval_batch"], meta["image"], seed=meta["eval_seed"])
    mirror = QuantContainer.load(g, GRAPHS / f"{NAME}.qjson", lib=_mirror_lib())
    env = mirror_env(mirror, x)
    qc = QuantContainer.load(g, GRAPHS / f"{NAME}.qjson", lib=gpu_lib)
    return qc, x, env, meta


def test_vit_b16_every_step_against_the_reference(vit_b16):
    from quantanything_b200.resident_vit import ResidentViT

    qc, x, env, meta = vit_b16
    net = ResidentViT(qc, meta["eval_batch"])
    kinds = [k for k, _ in net.steps]
    assert kinds.count("attention") == 12 and kinds.count("layernorm") == 25
    report = {}
    for i, kind, name, diff in teacher_forced(net, env, x, qc.graph.inputs[0].name):
        report[f"{i}:{kind}:{name}"] = (int(diff.max()), int((diff != 0).sum()), diff.size)
        if kind in INTEGER_KINDS:
            assert diff.max() == 0, (i, kind, name, int((diff != 0).sum()))
        elif kind in FALLBACK_KINDS:
            assert diff.max() <= FALLBACK_LSB, (i, kind, name, int(diff.max()))
            assert (diff != 0).sum() <= FALLBACK_FLIP_FRACTION * diff.size, (
                i, kind, name, int((diff != 0).sum()))
    checked = {k.split(":")[1] for k in report}
    assert set(INTEGER_KINDS + FALLBACK_KINDS) <= checked
    path = os.environ.get("QA_PARITY_REPORT")
    if path:
        flips = {kd: [sum(r[1] for k, r in report.items() if k.split(":")[1] == kd),
                      sum(r[2] for k, r in report.items() if k.split(":")[1] == kd)]
                 for kd in checked}
        with open(path, "w") as f:
            json.dump({"steps": report, "flips_by_kind": flips}, f, indent=1)


def test_vit_b16_logits_against_the_reference(vit_b16):
    from quantanything_b200.resident_vit import ResidentViT

    qc, x, env, meta = vit_b16
    net = ResidentViT(qc, meta["eval_batch"])
    net.forward_device(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    net.check_status()
    q = net.output_int().cpu().numpy().astype(np.int64)
    ref = np.load(GRAPHS / f"{NAME}.npz")["q"].astype(np.int64)
    mirror_out = np.asarray(env[qc.graph.outputs[0]]).astype(np.int64)
    np.testing.assert_array_equal(mirror_out.reshape(ref.shape), ref)  # mirror pinned
    diff = np.abs(q - ref)
    identical = float((diff == 0).mean())
    path = os.environ.get("QA_PARITY_REPORT")
    if path:
        with open(path + ".e2e.json", "w") as f:
            json.dump({"max_lsb": int(diff.max()), "identical": identical,
                       "argmax_equal": bool((q.argmax(1) == ref.argmax(1)).all())}, f)
    np.testing.assert_array_equal(q.argmax(1), ref.argmax(1))
    assert diff.max() <= E2E_MAX_LSB
    assert identical >= E2E_MIN_IDENTICAL
