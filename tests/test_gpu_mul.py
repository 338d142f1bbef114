"""Standalone Mul and BatchNorm layers on the resident executors (B200).

``networks.mul_mini`` keeps a SiLU as Sigmoid (a table layer) followed by
an integer Mul of two activations (quant_layers.py:516-540,
qa_kernels.cpp:334-345), so neither fuses into a convolution.  The graph is
calibrated on the C oracle and the same q.json runs on the GPU: the logits
must equal the oracle's layer-by-layer integer pass bit for bit, the
Softmax output within 1 LSB.
"""
import numpy as np
import pytest
import torch

from quantanything_b200 import networks
from quantanything_b200.container import QuantContainer

pytestmark = pytest.mark.gpu


def _logits_pass(qc, x):
    env = dict(qc.quantize_inputs({qc.graph.inputs[0].name: x}))
    for node in qc.graph.nodes:
        if node.op_type == "Softmax":
            return env, node.inputs[0]
        layer = qc.quant_layers[node.name]
        env.update(zip(node.outputs,
                       layer.quantized_infer_integer([env[n] for n in layer.data_inputs])))
    raise AssertionError("no Softmax")


@pytest.mark.parametrize("quant_type", ["int8", "uint8", "int16"])
def test_mul_mini_resident(gpu_lib, oracle, tmp_path, quant_type):
    from quantanything_b200.resident import ResidentNet
    from quantanything_b200.resident16 import ResidentNet16

    g = networks.mul_mini()
    qc = QuantContainer(g, quant_type, per_channel=True, lib=oracle)
    qc.calibrate([networks.images(4, 32, seed=s) for s in range(2)])
    path = tmp_path / f"mul_mini_{quant_type}.qjson"
    qc.save(path)
    # uint8 graphs run on the 16-bit route (their centred weights exceed int8)
    cls = ResidentNet if quant_type == "int8" else ResidentNet16
    net = cls(QuantContainer.load(g, path, lib=gpu_lib), 2)
    assert sum(kind == "mul" for kind, _ in net.steps) == 1
    x = networks.images(2, 32, seed=7)
    net.forward_device(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    net.check_status()
    q = net.out_q.cpu().numpy().astype(np.int64)
    assert np.abs(q - qc.run_integer_raw(x)).max() <= 1
    env, logits = _logits_pass(qc, x)
    got = net.tensor(logits).cpu().numpy().reshape(env[logits].shape)
    np.testing.assert_array_equal(got, env[logits])


@pytest.mark.parametrize("quant_type", ["int8", "uint8", "int16"])
def test_bn_mini_resident(gpu_lib, oracle, tmp_path, quant_type):
    """An unfolded BatchNormalization (negative gammas included: negative
    multipliers) as the per-channel requantize with a post-bias."""
    from quantanything_b200.resident import ResidentNet
    from quantanything_b200.resident16 import ResidentNet16

    g = networks.bn_mini()
    qc = QuantContainer(g, quant_type, per_channel=True, lib=oracle)
    qc.calibrate([networks.images(4, 32, seed=s) for s in range(2)])
    path = tmp_path / f"bn_mini_{quant_type}.qjson"
    qc.save(path)
    cls = ResidentNet if quant_type == "int8" else ResidentNet16
    net = cls(QuantContainer.load(g, path, lib=gpu_lib), 2)
    assert sum(kind == "bn" for kind, _ in net.steps) == 1
    x = networks.images(2, 32, seed=7)
    net.forward_device(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    net.check_status()
    q = net.out_q.cpu().numpy().astype(np.int64)
    assert np.abs(q - qc.run_integer_raw(x)).max() <= 1
    env, logits = _logits_pass(qc, x)
    got = net.tensor(logits).cpu().numpy().reshape(env[logits].shape)
    np.testing.assert_array_equal(got, env[logits])
