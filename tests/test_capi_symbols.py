"""The C-ABI library loads and exports every symbol include/moe_b200.h declares
(no compute call: this runs without a GPU)."""
import ctypes
import os
import re
import subprocess

from conftest import ROOT, load_package

HEADER = os.path.join(ROOT, "include", "moe_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^MOE_API[^;(]*?\b(moe_\w+)\s*\(", text, re.M)))


def test_header_declares_api():
    syms = declared_symbols()
    assert "moe_ffn_forward" in syms and "moe_tensor_mma_transposed_2x2" in syms
    assert len(syms) >= 20


def test_library_exports_every_declared_symbol():
    m = load_package()
    if not os.path.exists(m.LIB_PATH):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "llm.c_b200")], check=True)
    lib = ctypes.CDLL(m.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, f"not exported: {missing}"


def test_python_binding_covers_header():
    m = load_package()
    assert sorted(m.SIGNATURES) == declared_symbols()


def test_version_string_without_gpu():
    m = load_package()
    assert b"sm_100a" in m.lib().moe_version()
