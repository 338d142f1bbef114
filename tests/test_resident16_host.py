"""Host-side checks of the 16-bit entry points (CPU only, no kernel runs).

qa_conv16_fused_dev and qa_quantize_to_planes16_dev validate their
arguments before any CUDA call and report a clear error; the descriptors
below never reach a launch, so their (non-null, never dereferenced)
pointers are placeholders.
"""
import ctypes

import numpy as np
import pytest

from quantanything_b200 import native


@pytest.fixture(scope="module")
def lib():
    from quantanything_b200 import build
    from quantanything_b200.resident16 import device_api16

    lib = native.KernelLibrary(build.build())
    device_api16(lib)
    return lib


def _desc(**kw):
    from quantanything_b200.resident16 import FusedConv16Desc

    d = FusedConv16Desc()
    b = d.base
    b.x, b.x_pix_stride, b.x_signed, b.x_zp = 0x10000, 64, 1, 0
    b.N, b.H, b.W, b.C = 2, 8, 8, 64
    b.KH = b.KW = 3
    b.SH = b.SW = b.DH = b.DW = 1
    b.PH = b.PW = 1
    b.OH = b.OW = 8
    b.Cout, b.groups = 64, 1
    b.w, b.w_rows, b.w_kp = 0x20000, 64, 576
    b.mult, b.shift = 0x30000, 0x40000
    b.qmin, b.qmax = -32768, 32767
    b.out, b.out_pix_stride = 0x50000, 64
    b.block_n = 64
    d.x_plane = d.out_plane = 8192
    for k, v in kw.items():
        setattr(b if hasattr(b, k) else d, k, v)
    return d


def _call(lib, d):
    rc = lib.raw.qa_conv16_fused_dev(ctypes.byref(d), None)
    msg = lib.raw.qa_last_error().decode()
    lib.raw.qa_clear_error()
    return rc, msg


@pytest.mark.parametrize("field,value,words", [
    ("block_n", 48, "block_n"),
    ("x_signed", 0, "bad layout"),
    ("w_kp", 512, "bad layout"),          # shorter than K = 576
    ("w_rows", 32, "bad layout"),         # fewer rows than Cout
    ("C", 6, "bad layout"),               # channels per tap not a multiple of 4
    ("x_plane", 8194, "bad layout"),      # misaligned high plane
])
def test_conv16_rejects_bad_descriptors(lib, field, value, words):
    rc, msg = _call(lib, _desc(**{field: value}))
    assert rc != 0 and words in msg, msg


def test_conv16_rejects_k_beyond_exact_int32_partial_sums(lib):
    # K * 255 * 255 must stay below 2^31 for the three int32 accumulators
    k_ok = (2**31 - 1) // (255 * 255) // 4 * 4
    rc, msg = _call(lib, _desc(KH=1, KW=1, PH=0, PW=0, C=k_ok + 4, x_pix_stride=k_ok + 4,
                               w_kp=k_ok + 16))
    assert rc != 0 and "K too large" in msg, msg


def test_conv16_rejects_images_past_32bit_offsets(lib):
    rc, msg = _call(lib, _desc(H=8192, W=8192, OH=8192, OW=8192))
    assert rc != 0 and "image too large" in msg, msg


def test_grouped_conv16_rejects_uneven_groups(lib):
    rc, msg = _call(lib, _desc(groups=5, C=1, block_n=0))
    assert rc != 0 and "grouped" in msg, msg


def test_quantize_to_planes16_rejects_out_of_range_bounds(lib):
    rc = lib.raw.qa_quantize_to_planes16_dev(0x1000, 0x2000, 4096, 1, 3, 8, 8, 4, 0.1, 0,
                                             -32768, 40000, None)
    msg = lib.raw.qa_last_error().decode()
    lib.raw.qa_clear_error()
    assert rc != 0 and "qa_quantize_to_planes16_dev" in msg


@pytest.mark.parametrize("name", ["yolo_mini_uint16", "sppf_mini_uint16", "shaping_mini_uint16",
                                  "vit_mini_uint16"])
def test_uint16_shift_is_exact_through_the_integer_pass(oracle, name):
    """The uint16 resident route stores activations 32768 lower.  The
    shifted container (every activation zp / qmin / qmax / table moved by
    -32768) run through the drop-in integer pass gives the reference's
    outputs minus 32768, bit for bit, and the same dequantized floats."""
    import json

    from quantanything_b200 import networks
    from quantanything_b200.container import QuantContainer
    from quantanything_b200.resident16 import UINT16_SHIFT, shifted_container
    from tests.conftest import GOLDEN

    graphs = GOLDEN / "graphs"
    meta = json.loads((graphs / f"{name}.meta.json").read_text())
    g = getattr(networks, meta["builder"])(**meta["kwargs"])
    qc = QuantContainer.load(g, graphs / f"{name}.qjson", lib=oracle)
    x = networks.images(meta["eval_batch"], meta["image"], seed=meta["eval_seed"])
    ref = np.load(graphs / f"{name}.npz")
    sc = shifted_container(qc)  # the ViT's float fallbacks see (q - zp) only, too
    q = np.asarray(sc.run_integer_raw(x), np.int64)
    assert q.min() >= -UINT16_SHIFT and q.max() < UINT16_SHIFT
    np.testing.assert_array_equal(q + UINT16_SHIFT, ref["q"])
    y = sc.run_graph(x, "integer")
    np.testing.assert_array_equal(np.asarray(y).view(np.uint32), ref["y"].view(np.uint32))
    # the original container is untouched
    np.testing.assert_array_equal(np.asarray(qc.run_integer_raw(x)), ref["q"])
