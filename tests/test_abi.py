"""The C-ABI library builds for sm_100a, loads without a GPU, and exports every
entry point that include/*.h declares (no compute calls here)."""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\bAH_API\b[^;(]*?\b(ah_\w+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "ah_q4w_gemv" in names and "ah_dequant_q8_0_f32" in names and len(names) >= 30


def test_library_exports_every_declared_symbol():
    from agent_harness_b200 import _lib
    L = _lib.lib()
    missing = [n for n in declared_symbols() if not hasattr(L, n)]
    assert not missing, f"not exported: {missing}"


def test_python_signatures_cover_header():
    from agent_harness_b200 import _lib
    missing = [n for n in declared_symbols() if n not in _lib.SIGNATURES]
    assert not missing, f"no ctypes signature for: {missing}"


def test_sizes_without_gpu():
    # models/quantization.rs:423-435 — pure host arithmetic, no device needed
    from agent_harness_b200 import hostapi
    assert hostapi.packed_bytes(5) == 3
    assert hostapi.n_groups(65, 32) == 3
    assert hostapi.quantized_bytes(64, 32) == 2 * 4 + 32
    L = __import__("agent_harness_b200._lib", fromlist=["lib"]).lib()
    assert L.ah_strerror(-1) == b"invalid argument"


def test_product_path_does_not_touch_oracle():
    # The product package must never import or load the oracle.
    for py in glob.glob(os.path.join(ROOT, "agent_harness_b200", "**", "*.py"), recursive=True):
        src = open(py).read()
        assert "oracle" not in src, py
    for cu in glob.glob(os.path.join(ROOT, "agent_harness_b200", "csrc", "*")):
        assert "ah_oracle" not in open(cu).read(), cu
