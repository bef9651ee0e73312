"""One token through the single-row GEMV (gemv.cu's gemv_tc_kernel with the
token's K experts as row segments): gate/up rows of every slot in one
launch, down in column chunks, then the slot-order combine.  Checked
against the CPU oracle and against the fused layer kernel (MOE_NO_T1) on
the same layer; the routing is the five-launch path's, bit-exact."""
import numpy as np
import pytest

from test_gpu_moe import assert_output_close, assert_routing, build

pytestmark = pytest.mark.gpu

# (seed, d, d_ff, experts, top-k, qtype, renorm): the config-0 layer, Q4_0
# experts at a fused shape, the Mixtral structure at d_ff 2048, and a d_ff
# whose down rows take several column chunks (7168 = 7 x 1024)
SHAPES = {
    "olmoe_q8": (0, 2048, 1024, 64, 8, 1, False),
    "q4_top4": (31, 2048, 1024, 16, 4, 2, False),
    "wide_q4": (32, 4096, 2048, 8, 2, 2, True),
    "chunked_q4": (33, 1024, 7168, 4, 2, 2, True),
    "chunked_q8": (34, 1024, 7168, 4, 2, 1, False),
}


@pytest.fixture(scope="module")
def layers(orc):
    return {k: orc.make_layer(s, d, F, NE, K, qt, renorm=rn)
            for k, (s, d, F, NE, K, qt, rn) in SHAPES.items()}


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_t1_against_oracle_and_fused(moe, orc, layers, name, seed):
    L = layers[name]
    x = orc.make_tokens(500 + seed, 1, L["d_model"])
    ref, ids_ref, w_ref, _ = orc.moe_ffn(L, x)
    lay = build(moe, L, flags=moe.RENORM if L.get("renorm") else 0)
    try:
        got = lay.forward(x, flags=moe.FORCE_T1)
        ids, w, *_ = lay.routing(1)
        assert_routing(orc, x, L, 16, ids, w, ids_ref, w_ref)
        assert_output_close(got, ref)
        # the same token on the fused kernel: same routing, outputs within
        # the two kernels' rounding of the same sums
        fused = lay.forward(x, flags=moe.NO_T1)
        ids2, w2, *_ = lay.routing(1)
        np.testing.assert_array_equal(ids, ids2)
        np.testing.assert_array_equal(w, w2)
        scale = float(np.abs(ref).max())
        assert float(np.abs(got - fused).max()) <= 1e-5 * scale + 1e-7
        # repeatable bit for bit
        np.testing.assert_array_equal(lay.forward(x, flags=moe.FORCE_T1), got)
    finally:
        lay.close()


def test_t1_profiled_stages(moe, orc, layers):
    """MOE_PROFILE on the single-token path: the five stage times"""
    L = layers["wide_q4"]
    x = orc.make_tokens(510, 1, L["d_model"])
    lay = build(moe, L, flags=moe.RENORM)
    try:
        lay.forward(x, flags=moe.FORCE_T1 | moe.PROFILE)
        ms, n = lay.stage_ms()
        assert n == 1
        # router, top-k and dispatch are one launch: the routing stage is ~0
        assert all(v >= 0 for v in ms) and ms[0] > 0 and ms[2] > 0 and ms[3] > 0, ms
    finally:
        lay.close()


def test_t1_then_batches(moe, orc, layers):
    """one token between larger batches on the same layer: every result
    stays equal to the oracle's"""
    L = layers["q4_top4"]
    lay = build(moe, L)
    try:
        for T in (1, 5, 1, 40, 1):
            x = orc.make_tokens(520 + T, T, L["d_model"])
            ref, *_ = orc.moe_ffn(L, x)
            assert_output_close(lay.forward(x), ref)
    finally:
        lay.close()
