"""Import-time stand-in for the `onnx` package (absent in this container).

Only the fixture generator uses it: the reference's graph module imports
`onnx`, `onnx.helper` and `onnx.numpy_helper` at module level, but graphs
built directly as `OnnxGraph(Node ...)` never touch the protobuf API.
"""
import types as _types

helper = _types.ModuleType("onnx.helper")
numpy_helper = _types.ModuleType("onnx.numpy_helper")
shape_inference = _types.ModuleType("onnx.shape_inference")


class TensorProto:  # referenced only by type checks on attribute values
    pass


class ModelProto:
    pass
