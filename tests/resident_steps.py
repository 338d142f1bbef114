"""Test helpers: run a resident executor one step at a time, each step fed
the host mirror's tensors for its inputs (teacher forcing), so that every
kernel is compared with the reference on the reference's own inputs."""
import numpy as np
import torch


def mirror_env(qc, x):
    """Every tensor of the host mirror's integer pass (the reference's
    quantized_infer_integer per layer) on images ``x``."""
    from quantanything_b200 import float_ops

    env = qc.quantize_inputs(float_ops.normalize_feeds(qc.graph, x))
    for n in qc._const_names:
        env[n] = qc._const_q[n]
    for node in qc.graph.nodes:
        layer = qc.quant_layers[node.name]
        env.update(zip(node.outputs,
                       layer.quantized_infer_integer([env[n] for n in layer.data_inputs])))
    return env


def step_io(kind, payload):
    """(input pointers, output pointers) of one resident step."""
    if kind == "conv":
        d = payload.desc
        return [p for p in (d.x, d.res) if p], [p for p in (d.out, d.out2) if p]
    if kind in ("vit_embed", "gather", "attention"):
        return [payload[0].ptr], [payload[1].ptr]
    if kind == "layernorm":
        return [payload[1].ptr], [payload[2].ptr]
    if kind == "matmul_act":
        return [payload[1].ptr, payload[2].ptr], [payload[3].ptr]
    return [], []


def write_tensor(net, name, value):
    """Stores an int32 tensor (the mirror's layout of ``name``) into the
    executor's view of ``name`` (bytes, or the two byte planes of an int16
    tensor)."""
    v = net._views[name]
    rows = v.N * v.H * v.W
    src = np.asarray(value).reshape(v.N, v.C, v.H, v.W).transpose(0, 2, 3, 1).reshape(rows, v.C)
    # uint16 executors hold activations 32768 lower (net.tensor adds it back)
    src = src.astype(np.int64) - getattr(net, "_act_shift", 0)
    planes = [(0, 0)] if not v.plane else [(0, 0), (v.plane, 8)]  # (offset, bit shift)
    for off, shift in planes:
        dst = torch.as_strided(v.buf, (rows, v.C), (v.pix_stride, 1), v.offset + off)
        t = torch.from_numpy(
            np.ascontiguousarray((src.astype(np.int64) >> shift) & 0xFF).astype(np.uint8))
        dst.copy_(t.to(v.buf.device))


def run_step(net, step):
    saved = net.steps
    net.steps = [step]
    try:
        net.forward_device()
    finally:
        net.steps = saved
    torch.cuda.synchronize()
    net.check_status()


def teacher_forced(net, env, x, in_name, extra_inputs=None):
    """Runs every step of ``net`` on the mirror's inputs; yields (step index,
    kind, tensor name, absolute difference array) for every output the
    executor keeps under a name the mirror knows.  ``extra_inputs``: pointer
    -> view for operands that are not named views (transposed rows)."""
    by_ptr = {}
    for name, v in net._views.items():
        if name != in_name and name in env:
            by_ptr.setdefault(v.ptr, []).append(name)
    for name, v in (extra_inputs or {}).items():
        if name in env:
            by_ptr.setdefault(v.ptr, []).append(name)
    net.x_dev.copy_(torch.from_numpy(x))
    for i, (kind, payload) in enumerate(net.steps):
        ins, outs = step_io(kind, payload)
        for p in ins:
            if p in by_ptr:
                n0 = by_ptr[p][0]
                if n0 in net._views:
                    write_tensor(net, n0, env[n0])
        run_step(net, (kind, payload))
        for p in outs:
            for name in by_ptr.get(p, []):
                if name not in net._views:
                    continue
                got = net.tensor(name).cpu().numpy().reshape(-1).astype(np.int64)
                want = np.asarray(env[name]).reshape(-1).astype(np.int64)
                yield i, kind, name, np.abs(got - want)
