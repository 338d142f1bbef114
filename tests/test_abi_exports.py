"""The C-ABI library loads and exports every symbol the header declares.

CPU only: no compute call is made (there is no GPU in the build container).
"""
import ctypes
import re

import pytest

from quantanything_b200 import native
from tests.conftest import REPO

HEADER = REPO / "include" / "qa_kernels.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    names = re.findall(r"\b(qa_\w+)\s*\(", text)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib_path():
    from quantanything_b200 import build

    return build.build()


def test_header_declares_reference_abi():
    names = set(declared_functions())
    missing = set(native.REFERENCE_SIGNATURES) - names
    assert not missing, f"header lacks reference symbols {missing}"
    assert set(native.EXTENSION_SIGNATURES) <= names


def test_library_exports_every_declared_symbol(lib_path):
    lib = ctypes.CDLL(str(lib_path))
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_library_loads_through_wrapper(lib_path):
    lib = native.KernelLibrary(lib_path)
    assert lib.has_status
    assert lib.has_openmp() == 0
    assert lib.num_threads() >= 1


def test_reference_loader_signature_table_matches():
    """native.py's table is the reference loader's (native.py:104-128)."""
    sigs = native.REFERENCE_SIGNATURES
    assert len(sigs) == 17
    assert len(sigs["qa_conv_i32_i16_i32"][1]) == 19
    assert len(sigs["qa_requantize_i32"][1]) == 12
    assert len(sigs["qa_add"][1]) == 14


def test_fused_desc_layout_matches_header(tmp_path):
    """ctypes FusedConvDesc has the exact field offsets of the C struct."""
    import subprocess

    from quantanything_b200.resident import FusedConvDesc

    names = [f[0] for f in FusedConvDesc._fields_]
    src = tmp_path / "probe.c"
    src.write_text(
        '#include <stddef.h>\n#include <stdio.h>\n#include "qa_kernels.h"\nint main(void){\n'
        + "".join(f'printf("%zu\\n", offsetof(qa_fused_conv_desc, {n}));\n' for n in names)
        + 'printf("%zu\\n", sizeof(qa_fused_conv_desc));\nreturn 0;}\n')
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    want = [getattr(FusedConvDesc, n).offset for n in names] + [ctypes.sizeof(FusedConvDesc)]
    assert got == want


def test_fused16_desc_layout_matches_header(tmp_path):
    """ctypes FusedConv16Desc has the exact field offsets of the C struct."""
    import subprocess

    from quantanything_b200.resident16 import FusedConv16Desc

    names = [f[0] for f in FusedConv16Desc._fields_]
    src = tmp_path / "probe16.c"
    src.write_text(
        '#include <stddef.h>\n#include <stdio.h>\n#include "qa_kernels.h"\nint main(void){\n'
        + "".join(f'printf("%zu\\n", offsetof(qa_fused_conv16_desc, {n}));\n' for n in names)
        + 'printf("%zu\\n", sizeof(qa_fused_conv16_desc));\nreturn 0;}\n')
    exe = tmp_path / "probe16"
    subprocess.run(["gcc", "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    want = [getattr(FusedConv16Desc, n).offset for n in names] + [
        ctypes.sizeof(FusedConv16Desc)]
    assert got == want
