"""The C boundary's struct layout, checked by the C compiler: capi_harness.c
static-asserts that the reference's tensor_t (its own tensor.h, -DQ8_DOT as
the reference Makefile builds it) and moe_tensor_t have the same size, field
offsets and dtype values.  Runs where the reference sources are present."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.abspath(os.path.join(ROOT, "..", "reference"))


def test_tensor_t_layout_matches_moe_tensor_t():
    if not os.path.exists(os.path.join(REF, "tensor.h")):
        pytest.skip("reference sources absent")
    r = subprocess.run(["gcc", "-fsyntax-only", "-DFLASH_ATTENTION", "-DFUSED_GEMV", "-DQ8_DOT",
                        "-march=x86-64-v4", "-I" + REF, "-I" + os.path.join(ROOT, "include"),
                        os.path.join(ROOT, "oracle", "capi_harness.c")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
