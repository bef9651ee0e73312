"""The drop-in boundary from C: oracle/_ref/capi_harness is compiled against
the reference's own tensor.h (its static asserts pin tensor_t's size and
field offsets to moe_tensor_t's) and linked with the reference's sources and
libmoe_b200.so.  It runs the integration patch's moe_ffn body -- one
moe_ffn_forward (OLMoE, 3-D expert tensors) or moe_ffn_forward_split
(Mixtral, per-expert 2-D tensors, MOE_RENORM) call on tensor_t objects built
as gguf_tensor_3d/2d builds them -- and the reference's moe_ffn on the same
bytes.  Both outputs must agree within the tolerance, and with the oracle.

The harness is built where the reference sources are (build()); it travels
with the repository as a built file.  Skipped when it was not built.
"""
import os
import subprocess
import tempfile

import numpy as np
import pytest

from test_gpu_moe import MAX_ABS, REL_L2, rel_l2

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HARNESS = os.path.join(ROOT, "oracle", "_ref", "capi_harness")


@pytest.mark.parametrize("case", [
    (5, 2048, 1024, 16, 4, 1, 0, 81),    # OLMoE layout, Q8_0, T = 5 (fused kernel)
    (70, 2048, 1024, 16, 4, 1, 0, 82),   # 70 tokens: the grouped GEMM path
    (3, 4096, 2048, 8, 2, 2, 1, 83),     # Mixtral layout (per-expert tensors), Q4_0, renorm
])
def test_c_caller_with_reference_tensor_t(orc, case):
    if not os.path.exists(HARNESS):
        pytest.skip("oracle/_ref/capi_harness not built (reference sources absent at build)")
    T, d, F, NE, K, qt, renorm, seed = case
    L = orc.make_layer(seed, d, F, NE, K, qt, renorm=bool(renorm))
    x = orc.make_tokens(seed, T, d)
    with tempfile.TemporaryDirectory() as td:
        for name, arr in (("x", x), ("router", L["router_w"]), ("gate", L["gate"]),
                          ("up", L["up"]), ("down", L["down"])):
            np.ascontiguousarray(arr).tofile(os.path.join(td, name + ".bin"))
        r = subprocess.run([HARNESS, td, str(T), str(d), str(F), str(NE), str(K), str(qt),
                            str(renorm)], capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
        got = np.fromfile(os.path.join(td, "out_gpu.bin"), np.float32).reshape(T, d)
        ref = np.fromfile(os.path.join(td, "out_ref.bin"), np.float32).reshape(T, d)
    assert float(np.abs(got - ref).max()) <= MAX_ABS
    assert rel_l2(got, ref) <= REL_L2
    orc_out = orc.moe_ffn(L, x)[0]
    assert rel_l2(got, orc_out) <= REL_L2
