"""Runs the reference's own, unchanged Python package on top of a kernel
library loaded through the reference's QA_LIB switch (test helper).

The reference package (``quantization``, as ``pip install --target
baseline/_ref`` puts it; any directory holding it can be named with
``QA_REFERENCE_PKG``) is imported with the import stub for the absent
``onnx`` module.  Its loader (quantization/native.py:104-145) opens
``QA_LIB`` with ctypes and declares every entry point's restype / argtypes
itself; a missing symbol there would silently fall back to NumPy, so the
script checks that the library really loaded.

Modes (one JSON object on stdout):
  signatures  -- the restype / argtypes the reference's loader declared on
                 the library (no compute call: runs without a GPU)
  graphs      -- the reference's QuantContainer (quant_container.py) loads
                 each golden fixture's q.json and runs its integer pass
                 (``_execute(x, "integer")``), every layer calling the
                 library; reports whether the int32 output and the
                 dequantized float32 output equal the reference-generated
                 fixture bit for bit, plus a few direct calls of the
                 reference's native.* wrappers against exact int64 NumPy.

    python tests/reference_dropin.py <mode> <library path>
"""
import ctypes
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
GRAPHS = HERE / "golden" / "graphs"
GRAPH_CASES = ["yolo_mini_int8", "yolo_mini_uint8", "yolo_mini_int16", "sppf_mini_int8",
               "vit_mini_int8", "vit_mini_int16", "yolov8n_cls_int8"]


def reference_package_dir():
    """Directory holding the reference's ``quantization`` package, or None."""
    cand = os.environ.get("QA_REFERENCE_PKG") or str(REPO / "baseline" / "_ref")
    return cand if (Path(cand) / "quantization" / "native.py").exists() else None


def _import_reference(lib_path):
    pkg = reference_package_dir()
    if pkg is None:
        raise SystemExit("reference package not found")
    os.environ["QA_LIB"] = str(lib_path)
    sys.path[:0] = [str(HERE / "golden" / "_onnx_stub"), pkg, str(REPO)]
    from quantization import native

    if not native.available():
        raise SystemExit(f"the reference's loader did not load {lib_path}: "
                         f"{native.load_error()}")
    return native


def _type_name(t):
    return None if t is None else t.__name__


def signatures(lib_path):
    native = _import_reference(lib_path)
    names = ["qa_num_threads", "qa_set_num_threads", "qa_has_openmp", "qa_gemm_f32",
             "qa_gemm_i16_i32", "qa_gemm_i32_i64", "qa_conv_f32", "qa_conv_i32_i16_i32",
             "qa_conv_i32_i32_i64", "qa_requantize_i32", "qa_requantize_i64", "qa_rescale",
             "qa_add", "qa_mul", "qa_lut", "qa_quantize_f32", "qa_dequantize_f32"]
    out = {}
    for n in names:
        fn = getattr(native._lib, n)
        out[n] = [_type_name(fn.restype), [_type_name(a) for a in (fn.argtypes or [])]]
    return {"library": str(lib_path), "declared": out}


def graphs(lib_path):
    native = _import_reference(lib_path)
    from quantization import QuantContainer

    from quantanything_b200 import networks
    from tests.golden.graph_fixtures import to_reference_graph

    res = {"library": str(lib_path), "graphs": {}, "kernels": {}}
    for name in GRAPH_CASES:
        meta = json.loads((GRAPHS / f"{name}.meta.json").read_text())
        g = getattr(networks, meta["builder"])(**meta["kwargs"])
        rg = to_reference_graph(g)
        qc = QuantContainer.load(rg, GRAPHS / f"{name}.qjson")
        x = networks.images(meta["eval_batch"], meta["image"], seed=meta["eval_seed"])
        env, out = qc._execute(x, "integer")
        want = np.load(GRAPHS / f"{name}.npz")
        q = np.asarray(env[rg.outputs[0]], np.int32)
        res["graphs"][name] = {
            "int_equal": bool(np.array_equal(q, want["q"])),
            "float_equal": bool(np.array_equal(np.asarray(out, np.float32).view(np.uint32),
                                               want["y"].view(np.uint32)))}
    rng = np.random.default_rng(0)
    a = rng.integers(-(2**15), 2**15, (70, 300)).astype(np.int64)
    b = rng.integers(-(2**15), 2**15, (300, 90)).astype(np.int64)
    exact = a @ b
    res["kernels"]["gemm_int narrow"] = bool(np.array_equal(
        native.gemm_int(a, b, wide=False).astype(np.int64),
        ((exact + 2**31) % 2**32 - 2**31)))
    res["kernels"]["gemm_int wide"] = bool(np.array_equal(
        native.gemm_int(a, b, wide=True).astype(np.int64), exact))
    x = rng.integers(-128, 128, (2, 16, 9, 9)).astype(np.int64)
    w = rng.integers(-127, 128, (8, 16, 3, 3)).astype(np.int64)
    y = native.conv2d_int(x, w, (1, 1), (1, 1, 1, 1), (1, 1), 1, wide=True)
    xp = np.pad(x, ((0, 0), (0, 0), (1, 1), (1, 1)))
    cols = np.stack([xp[:, :, i:i + 9, j:j + 9] for i in range(3) for j in range(3)], 2)
    ref = np.einsum("nckhw,ock->nohw", cols, w.reshape(8, 16, 9))
    res["kernels"]["conv2d_int wide"] = bool(np.array_equal(np.asarray(y, np.int64), ref))
    return res


if __name__ == "__main__":
    mode, lib = sys.argv[1], sys.argv[2]
    print(json.dumps({"signatures": signatures, "graphs": graphs}[mode](lib)))
