"""Seeded random-init graphs of the benchmark networks.

No checkpoints or datasets are reachable, so the benchmark networks are
built directly as graphs with random weights of the right architecture,
already in the form the reference's load-time passes produce
(graph_passes.py): BatchNorm folded into the preceding Conv, and
``x * sigmoid(x)`` collapsed into one ``FusedElementwise`` node that the
quantizer turns into a lookup table.

* :func:`yolov8n_cls` -- YOLOv8n-cls (ultralytics ``yolov8n-cls.yaml`` at
  depth 0.33 / width 0.25): Conv 3x3 s2 16, Conv 3x3 s2 32, C2f(32, n=1),
  Conv s2 64, C2f(64, n=2), Conv s2 128, C2f(128, n=2), Conv s2 256,
  C2f(256, n=1), Conv 1x1 1280, GlobalAveragePool, Linear 1000, Softmax;
  every conv followed by SiLU; C2f bottlenecks with residual adds.
* :func:`yolo_mini` -- the small YOLO-like test graph shape of the
  reference's test-suite (stem, C2f-style split/add/concat, depthwise +
  pointwise, GAP, Gemm, Softmax) at a configurable width.
* :func:`vit` -- a Vision Transformer (ViT-B/16 at full size) in the
  reference's post-pass form.
"""

import numpy as np

from quantanything_b200.graph import Graph, Node, ValueInfo


class GraphBuilder:
    """Accumulates nodes and initializers with unique names."""

    def __init__(self, seed=0):
        self.rng = np.random.default_rng(seed)
        self.nodes, self.inits, self._n = [], {}, 0

    def name(self, base):
        self._n += 1
        return f"{base}_{self._n}"

    def const(self, value, base="const"):
        n = self.name(base)
        self.inits[n] = np.asarray(value)
        return n

    def op(self, op_type, inputs, n_out=1, **attrs):
        outs = [self.name(op_type.lower()) for _ in range(n_out)]
        self.nodes.append(Node(self.name(op_type), op_type, list(inputs), outs, attrs))
        return outs[0] if n_out == 1 else outs

    def conv(self, x, cin, cout, k=3, stride=1, pad=None, groups=1, bn=True):
        """Conv with He-normal weights; a random inference BatchNorm is
        folded in (w * gamma/sqrt(var+eps), bias beta - mean*gamma/sqrt(..))."""
        pad = k // 2 if pad is None else pad
        fan_in = (cin // groups) * k * k
        w = self.rng.standard_normal((cout, cin // groups, k, k)) * np.sqrt(2.0 / fan_in)
        if bn:
            gamma = self.rng.uniform(0.5, 1.5, cout)
            beta = self.rng.normal(0.0, 0.1, cout)
            mean = self.rng.normal(0.0, 0.1, cout)
            var = self.rng.uniform(0.5, 1.5, cout)
            a = gamma / np.sqrt(var + 1e-3)
            w = w * a.reshape(-1, 1, 1, 1)
            b = beta - mean * a
        else:
            b = self.rng.normal(0.0, 0.05, cout)
        return self.op("Conv", [x, self.const(w.astype(np.float32), "w"),
                                self.const(b.astype(np.float32), "b")],
                       kernel_shape=[k, k], strides=[stride, stride], pads=[pad] * 4,
                       dilations=[1, 1], group=groups)

    def silu(self, x):
        """x * sigmoid(x) as the fused element-wise node the reference's
        fusion pass emits (graph_passes.py:208-272)."""
        s = self.name("sigmoid")
        y = self.name("silu")
        sub = [Node(self.name("Sigmoid"), "Sigmoid", [x], [s]),
               Node(self.name("Mul"), "Mul", [x, s], [y])]
        self.nodes.append(Node(self.name("SiLU") + "_fused", "FusedElementwise", [x], [y],
                               {"nodes": sub, "consts": {}}))
        return y

    def conv_silu(self, x, cin, cout, k=3, stride=1, groups=1):
        return self.silu(self.conv(x, cin, cout, k, stride, groups=groups))

    def c2f(self, x, c1, c2, n=1, shortcut=True):
        """C2f block: cv1 1x1 -> split in halves -> n bottlenecks (two 3x3
        conv-SiLU, residual add) -> concat of all branches -> cv2 1x1."""
        c = c2 // 2
        y = self.conv_silu(x, c1, 2 * c, 1)
        a, b = self.op("Split", [y, self.const(np.array([c, c], np.int64), "split")], n_out=2,
                       axis=1)
        branches, cur = [a, b], b
        for _ in range(n):
            t = self.conv_silu(cur, c, c, 3)
            t = self.conv_silu(t, c, c, 3)
            cur = self.op("Add", [cur, t]) if shortcut else t
            branches.append(cur)
        y = self.op("Concat", branches, axis=1)
        return self.conv_silu(y, (2 + n) * c, c2, 1)

    def head(self, x, cin, classes, hidden=None):
        if hidden:
            x = self.conv_silu(x, cin, hidden, 1)
            cin = hidden
        x = self.op("GlobalAveragePool", [x])
        x = self.op("Flatten", [x], axis=1)
        std = np.sqrt(1.0 / cin)
        w = (self.rng.standard_normal((classes, cin)) * std).astype(np.float32)
        b = self.rng.normal(0.0, 0.05, classes).astype(np.float32)
        x = self.op("Gemm", [x, self.const(w, "fc_w"), self.const(b, "fc_b")], transB=1)
        return self.op("Softmax", [x], axis=1)

    def build(self, input_name, input_shape, output):
        return Graph(self.nodes, self.inits, [ValueInfo(input_name, list(input_shape))],
                     [output])


def yolov8n_cls(seed=0, classes=1000, image=224):
    """YOLOv8n-cls graph with random init (BN folded, SiLU fused)."""
    b = GraphBuilder(seed)
    x = "images"
    y = b.conv_silu(x, 3, 16, 3, 2)
    y = b.conv_silu(y, 16, 32, 3, 2)
    y = b.c2f(y, 32, 32, 1)
    y = b.conv_silu(y, 32, 64, 3, 2)
    y = b.c2f(y, 64, 64, 2)
    y = b.conv_silu(y, 64, 128, 3, 2)
    y = b.c2f(y, 128, 128, 2)
    y = b.conv_silu(y, 128, 256, 3, 2)
    y = b.c2f(y, 256, 256, 1)
    y = b.head(y, 256, classes, hidden=1280)
    return b.build(x, ["N", 3, image, image], y)


def yolo_mini(seed=0, size=32, classes=10, width=16):
    """Small YOLO-like graph: stem, C2f-style split/add/concat, depthwise +
    pointwise, GAP, Gemm, Softmax (the reference test-suite's structure)."""
    b = GraphBuilder(seed)
    x = "images"
    y = b.conv_silu(x, 3, width, 3, 2)
    y = b.conv_silu(y, width, 2 * width, 3, 2)
    a, c = b.op("Split", [y, b.const(np.array([width, width], np.int64), "split")], n_out=2,
                axis=1)
    d = b.conv_silu(c, width, width, 3)
    d = b.op("Add", [c, b.conv_silu(d, width, width, 3)])
    y = b.op("Concat", [a, c, d], axis=1)
    y = b.conv_silu(y, 3 * width, 4 * width, 1)
    y = b.conv_silu(y, 4 * width, 4 * width, 3, groups=4 * width)
    y = b.conv_silu(y, 4 * width, 8 * width, 1)
    y = b.head(y, 8 * width, classes)
    return b.build(x, ["N", 3, size, size], y)


def sppf_mini(seed=0, size=32, classes=10, width=16):
    """Small graph with a YOLOv8 SPPF block (three chained MaxPool k5 s1 p2
    whose outputs are concatenated), exercising integer MaxPool padded with
    qmin (quant_layers.py:647-648)."""
    b = GraphBuilder(seed)
    x = "images"
    y = b.conv_silu(x, 3, width, 3, 2)
    y = b.conv_silu(y, width, 2 * width, 3, 2)
    c = b.conv_silu(y, 2 * width, width, 1)
    pools = [c]
    for _ in range(3):
        pools.append(b.op("MaxPool", [pools[-1]], kernel_shape=[5, 5], strides=[1, 1],
                          pads=[2, 2, 2, 2]))
    y = b.op("Concat", pools, axis=1)
    y = b.conv_silu(y, 4 * width, 2 * width, 1)
    y = b.head(y, 2 * width, classes)
    return b.build(x, ["N", 3, size, size], y)


def mul_mini(seed=0, size=32, classes=10, width=16):
    """Small graph whose activations stay unfused: Sigmoid (a table) and an
    activation x activation Mul, i.e. SiLU as the graph holds it before the
    reference's element-wise fusion pass (graph_passes.py:208-272), so the
    integer Mul layer (quant_layers.py:516-540) runs on its own."""
    b = GraphBuilder(seed)
    x = "images"
    y = b.conv_silu(x, 3, width, 3, 2)
    y = b.conv(y, width, 2 * width, 3, 2)
    y = b.op("Mul", [y, b.op("Sigmoid", [y])])
    y = b.conv_silu(y, 2 * width, 2 * width, 3)
    y = b.head(y, 2 * width, classes)
    return b.build(x, ["N", 3, size, size], y)


def bn_mini(seed=0, size=32, classes=10, width=16):
    """Small graph with an unfolded inference BatchNormalization after a
    bias-free conv (some channels with negative gamma), i.e. the integer
    BatchNorm layer (quant_layers.py:405-441) running on its own."""
    b = GraphBuilder(seed)
    x = "images"
    y = b.conv_silu(x, 3, width, 3, 2)
    y = b.conv(y, width, 2 * width, 3, 2, bn=False)
    c = 2 * width
    gamma = b.rng.uniform(0.5, 1.5, c) * np.where(np.arange(c) % 5 == 0, -1.0, 1.0)
    params = [gamma, b.rng.normal(0.0, 0.1, c), b.rng.normal(0.0, 0.1, c),
              b.rng.uniform(0.5, 1.5, c)]
    y = b.op("BatchNormalization", [y] + [b.const(v.astype(np.float32), "bn") for v in params],
             epsilon=1e-3)
    y = b.silu(y)
    y = b.conv_silu(y, 2 * width, 2 * width, 3)
    y = b.head(y, 2 * width, classes)
    return b.build(x, ["N", 3, size, size], y)


def shaping_mini(seed=0, size=32, classes=10, width=16):
    """Small graph with the reference's scale-preserving layout operators on
    activations (quant_layers.py:593-650): an asymmetric zero-point Pad in
    front of an unpadded conv, spatial Transposes, a channel Slice on a
    16-channel boundary, a strided spatial Slice, an unaligned channel Slice
    and a channel Pad."""
    b = GraphBuilder(seed)
    i64 = np.int64
    x = "images"
    y = b.conv_silu(x, 3, width, 3, 2)                                   # [N, w, s/2, s/2]
    y = b.op("Pad", [y, b.const(np.array([0, 0, 1, 2, 0, 0, 2, 1], i64), "pads")],
             mode="constant")                                             # H, W + 3
    y = b.silu(b.conv(y, width, 2 * width, 3, 1, pad=0))                  # H, W + 1
    y = b.op("Transpose", [y], perm=[0, 1, 3, 2])
    y = b.op("Slice", [y, b.const(np.array([width], i64), "starts"),
                       b.const(np.array([2 * width], i64), "ends"),
                       b.const(np.array([1], i64), "axes")])              # channels w .. 2w
    y = b.conv_silu(y, width, width, 3)
    y = b.op("Slice", [y, b.const(np.array([1, 0], i64), "starts"),
                       b.const(np.array([2**63 - 1, size // 2], i64), "ends"),
                       b.const(np.array([2, 3], i64), "axes"),
                       b.const(np.array([2, 1], i64), "steps")])          # rows 1::2, cols :s/2
    y = b.op("Transpose", [y], perm=[0, 1, 3, 2])
    y = b.op("Slice", [y, b.const(np.array([4], i64), "starts"),
                       b.const(np.array([4 + width // 2], i64), "ends"),
                       b.const(np.array([1], i64), "axes")])              # w/2 channels from 4
    y = b.op("Pad", [y, b.const(np.array([0, 2, 0, 0, 0, width // 2 - 2, 0, 0], i64), "pads")],
             mode="constant")                                             # back to w channels
    y = b.conv_silu(y, width, 2 * width, 3, 2)
    y = b.head(y, 2 * width, classes)
    return b.build(x, ["N", 3, size, size], y)


def vit(seed=0, img=32, patch=8, dim=32, heads=4, depth=2, classes=10, batch=4, mlp=4,
        std=None, attention="heads"):
    """A Vision Transformer in the reference's post-pass form (the structure
    of its ``build_vit`` test model after graph_passes.py): patch-embedding
    Conv -> Reshape -> Transpose, a constant cls token concatenated in front
    (the batch Expand folded), a positional-embedding Add, ``depth`` pre-LN
    blocks (LayerNormalization; MatMul with the bias as third input; head
    split by Reshape / Transpose / Split / Squeeze; activation x activation
    MatMuls, the 1/sqrt(head_dim) Mul and Softmax; GELU as one fused
    element-wise erf chain), the cls token gathered before the final
    LayerNormalization, and a Gemm head.  The batch is static (it appears in
    the Reshape shapes).  ``std``: weight init (trunc-normal-like, default
    1/sqrt(fan_in); ViT-B/16 uses 0.02).

    ``vit(img=224, patch=16, dim=768, heads=12, depth=12, classes=1000,
    batch=B, std=0.02)`` is ViT-B/16.

    ``attention="gram"`` replaces each block's multi-head attention by plain
    activation x activation MatMuls on the token rows (no head split, no
    Softmax): S = MatMul(q, Transpose(k, [0, 2, 1])), O = MatMul(S, v), then
    the projection and residual Add -- a graph whose act x act MatMuls are
    the reference's stand-alone float fallbacks (quant_layers.py:195-205)."""
    b = GraphBuilder(seed)
    rng = b.rng
    hd = dim // heads
    grid = img // patch
    tokens = grid * grid + 1
    f32 = np.float32

    def weight(fan_in, shape):
        s_ = std if std is not None else 1.0 / np.sqrt(fan_in)
        return np.clip(rng.standard_normal(shape), -2, 2).astype(f32) * f32(s_)

    def linear(x, cin, cout):
        w = b.const(weight(cin, (cin, cout)), "w")
        bias = b.const(rng.normal(0.0, 0.02, cout).astype(f32), "b")
        return b.op("MatMul", [x, w, bias])

    def layer_norm(x):
        # the reference's passes move the LayerNorm gain into the next linear
        # layer; random-init gains are 1 and shifts 0
        return b.op("LayerNormalization", [x, b.const(np.ones(dim, f32), "ln_g"),
                                           b.const(np.zeros(dim, f32), "ln_b")],
                    axis=-1, epsilon=1e-6)

    def gelu(x):
        d, e, a, m, y = (b.name(t) for t in ("div", "erf", "add", "mul", "gelu"))
        sub = [Node(b.name("Div"), "Div", [x, "sqrt2"], [d]),
               Node(b.name("Erf"), "Erf", [d], [e]),
               Node(b.name("Add"), "Add", [e, "one"], [a]),
               Node(b.name("Mul"), "Mul", [x, a], [m]),
               Node(b.name("Mul"), "Mul", [m, "half"], [y])]
        consts = {"sqrt2": np.float32(np.sqrt(2.0)), "one": np.float32(1.0),
                  "half": np.float32(0.5)}
        b.nodes.append(Node(b.name("GELU") + "_fused", "FusedElementwise", [x], [y],
                            {"nodes": sub, "consts": consts}))
        return y

    pw = weight(3 * patch * patch, (dim, 3, patch, patch))
    x = b.op("Conv", ["images", b.const(pw, "w"), b.const(rng.normal(0, 0.02, dim).astype(f32),
                                                           "b")],
             kernel_shape=[patch, patch], strides=[patch, patch], pads=[0, 0, 0, 0],
             dilations=[1, 1], group=1)
    x = b.op("Reshape", [x, b.const(np.array([batch, dim, -1], np.int64), "shape")])
    x = b.op("Transpose", [x], perm=[0, 2, 1])
    cls = np.broadcast_to(rng.normal(0.0, 0.1, (1, 1, dim)), (batch, 1, dim)).astype(f32)
    x = b.op("Concat", [b.const(np.ascontiguousarray(cls), "cls"), x], axis=1)
    x = b.op("Add", [x, b.const(rng.normal(0.0, 0.1, (1, tokens, dim)).astype(f32), "pos")])
    for _ in range(depth):
        h = layer_norm(x)
        if attention == "gram":
            q, k, v = linear(h, dim, dim), linear(h, dim, dim), linear(h, dim, dim)
            s_ = b.op("MatMul", [q, b.op("Transpose", [k], perm=[0, 2, 1])])
            o = b.op("MatMul", [s_, v])
            x = b.op("Add", [x, linear(o, dim, dim)])
            h = gelu(linear(layer_norm(x), dim, mlp * dim))
            x = b.op("Add", [x, linear(h, mlp * dim, dim)])
            continue
        qkv = linear(h, dim, 3 * dim)
        qkv = b.op("Reshape", [qkv, b.const(np.array([batch, tokens, 3, heads, hd], np.int64),
                                             "shape")])
        qkv = b.op("Transpose", [qkv], perm=[2, 0, 3, 1, 4])
        parts = b.op("Split", [qkv], n_out=3, axis=0)
        q, k, v = [b.op("Squeeze", [t, b.const(np.array([0], np.int64), "axes")])
                   for t in parts]
        att = b.op("MatMul", [q, b.op("Transpose", [k], perm=[0, 1, 3, 2])])
        att = b.op("Mul", [att, b.const(np.float32(hd ** -0.5), "scale")])
        att = b.op("Softmax", [att], axis=-1)
        o = b.op("Transpose", [b.op("MatMul", [att, v])], perm=[0, 2, 1, 3])
        o = b.op("Reshape", [o, b.const(np.array([batch, tokens, dim], np.int64), "shape")])
        x = b.op("Add", [x, linear(o, dim, dim)])
        h = gelu(linear(layer_norm(x), dim, mlp * dim))
        x = b.op("Add", [x, linear(h, mlp * dim, dim)])
    x = b.op("Gather", [x, b.const(np.array(0, np.int64), "index")], axis=1)
    x = layer_norm(x)
    w = weight(dim, (classes, dim))
    y = b.op("Gemm", [x, b.const(w, "head_w"), b.const(rng.normal(0, 0.02, classes).astype(f32),
                                                        "head_b")], transB=1)
    return b.build("images", [batch, 3, img, img], y)


def images(n, size=224, seed=1):
    """N(0, 1) pixels clipped to +-3 (the configuration's input distribution)."""
    rng = np.random.default_rng(seed)
    return np.clip(rng.standard_normal((n, 3, size, size)), -3, 3).astype(np.float32)
