"""The reference's own loader accepts the CUDA library as a drop-in (CPU).

tests/reference_dropin.py imports the reference's unchanged package with
QA_LIB pointing at libqa_kernels.so; the reference's loader
(quantization/native.py:104-145) must load it -- every one of its 17
symbols resolved -- and the restype / argtypes it declares must be exactly
the signature table this package declares (native.REFERENCE_SIGNATURES).
No compute call is made, so no GPU is needed.  Skipped when the reference
package is not installed (baseline/_ref, or QA_REFERENCE_PKG).
"""
import json
import subprocess
import sys

import pytest

from quantanything_b200 import native
from tests.conftest import REPO
from tests.reference_dropin import reference_package_dir


def _name(t):
    return None if t is None else t.__name__


@pytest.mark.skipif(reference_package_dir() is None, reason="reference package not installed")
def test_reference_loader_declares_our_table_on_the_cuda_library():
    from quantanything_b200 import build

    lib = build.build()
    proc = subprocess.run([sys.executable, str(REPO / "tests" / "reference_dropin.py"),
                           "signatures", str(lib)], capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-2000:]
    got = json.loads(proc.stdout.strip().splitlines()[-1])["declared"]
    ours = {n: [_name(r), [_name(a) for a in args]]
            for n, (r, args) in native.REFERENCE_SIGNATURES.items()}
    assert got == ours
