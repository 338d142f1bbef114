"""Minimal graph IR: the in-memory form the reference builds from ONNX.

Mirrors the reference's ``OnnxGraph`` / ``Node`` (quantization/onnx_graph.py
:17-35, :91-269) for graphs constructed directly in memory: a topologically
ordered node list, a dict of constant initializers, graph inputs and
outputs.  Loading ``.onnx`` protobufs and the load-time rewrite passes are
outside the hot path and are not part of this package; graphs arrive already
in the post-pass form (Conv with folded BatchNorm, element-wise chains as
``FusedElementwise``).
"""

from collections import defaultdict, deque
from dataclasses import dataclass, field


@dataclass
class Node:
    """One operator instance (onnx_graph.py:17-35)."""

    name: str
    op_type: str
    inputs: list
    outputs: list
    attrs: dict = field(default_factory=dict)

    def attr(self, key, default=None):
        return self.attrs.get(key, default)


@dataclass
class ValueInfo:
    """A graph input: name, (possibly symbolic) shape, dtype."""

    name: str
    shape: list
    dtype: object = None


class Graph:
    """Topologically sorted graph with constants resolved to NumPy."""

    def __init__(self, nodes, initializers, inputs, outputs, opset=13):
        self.nodes = list(nodes)
        self.initializers = dict(initializers)
        self.inputs = [i if isinstance(i, ValueInfo) else ValueInfo(i, []) for i in inputs]
        self.outputs = list(outputs)
        self.opset = opset
        self.toposort()

    def _index(self):
        self.producers = {}
        self.consumers = defaultdict(list)
        for node in self.nodes:
            for out in node.outputs:
                self.producers[out] = node
            for inp in node.inputs:
                if inp:
                    self.consumers[inp].append(node)

    def toposort(self):
        """Kahn ordering; raises on cycles or undefined tensors
        (onnx_graph.py:237-259)."""
        ready_names = set(self.initializers) | {v.name for v in self.inputs}
        indeg, waiting = {}, defaultdict(list)
        for idx, node in enumerate(self.nodes):
            missing = {i for i in node.inputs if i and i not in ready_names}
            indeg[idx] = len(missing)
            for m in missing:
                waiting[m].append(idx)
        queue = deque(i for i, d in indeg.items() if d == 0)
        order = []
        while queue:
            idx = queue.popleft()
            order.append(idx)
            for out in self.nodes[idx].outputs:
                for j in waiting.get(out, []):
                    indeg[j] -= 1
                    if indeg[j] == 0:
                        queue.append(j)
        if len(order) != len(self.nodes):
            raise ValueError("graph has a cycle or an undefined tensor")
        self.nodes = [self.nodes[i] for i in order]
        self._index()

    def is_constant(self, name):
        return name in self.initializers

    @property
    def input_names(self):
        return [v.name for v in self.inputs]
