"""The prefill grouped GEMM (tcgen05, TMEM accumulators) against the CPU
oracle, and against the decode expert kernels at sizes where running the
oracle would take too long.

Batches of more than 64 tokens take the GEMM when the layer's shapes allow
it (rows a multiple of 128, columns a multiple of 256); MOE_FORCE_GEMM
selects it for any batch, MOE_FORCE_GEMV never.  The GEMM splits weights
(d * q) and activations into fp16 hi + lo and sums three tensor-core
products (hi x hi, hi x lo, lo x hi) in fp32, so it is held to the
north-star tolerance and, tighter, to rel-L2 1e-4 / max-abs 2e-4 of the fp32
oracle.  One fp16 term per operand would reach ~5e-4 rel-L2; what remains
with three terms (1.8e-5 rel-L2 on config 0) is the tensor cores' fp32
accumulation, which truncates instead of rounding.
"""
TIGHT_ABS, TIGHT_REL = 2e-4, 1e-4
import numpy as np
import pytest

from test_gpu_moe import assert_dispatch, assert_output_close, assert_routing, build, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def olmoe(orc):
    return orc.make_layer(0, 2048, 1024, 64, 8, orc.Q8_0)


@pytest.fixture(scope="module")
def q4_layer(orc):
    return orc.make_layer(33, 2048, 1024, 16, 4, orc.Q4_0, zipf=True)


def check_vs_oracle(moe, orc, L, x, flags=0):
    T = x.shape[0]
    ref, ids_ref, w_ref, _ = orc.moe_ffn(L, x)
    lay = build(moe, L, flags=moe.RENORM if L.get("renorm") else 0)
    got = lay.forward(x, flags=flags)
    ids, w, counts, offsets, perm = lay.routing(T)
    assert_routing(orc, x, L, 16, ids, w, ids_ref, w_ref)
    assert_dispatch(orc, ids, counts, offsets, perm, L["n_experts"])
    assert_output_close(got, ref)
    assert float(np.abs(got - ref).max()) <= TIGHT_ABS
    assert rel_l2(got, ref) <= TIGHT_REL
    lay.close()
    return got, ref


@pytest.mark.parametrize("T", [65, 257])
def test_gemm_config0(moe, orc, olmoe, T):
    check_vs_oracle(moe, orc, olmoe, orc.make_tokens(90 + T, T, 2048))


@pytest.mark.parametrize("T", [1, 17, 64])
def test_gemm_forced_small_batches(moe, orc, olmoe, T):
    """partial pair tiles and experts with one or two pairs"""
    check_vs_oracle(moe, orc, olmoe, orc.make_tokens(95 + T, T, 2048), flags=moe.FORCE_GEMM)


def test_gemm_q4_0_zipf(moe, orc, q4_layer):
    """Q4_0 experts; the Zipf bias sends hundreds of pairs to a few experts
    (several 128-pair tiles per expert)"""
    check_vs_oracle(moe, orc, q4_layer, orc.make_tokens(97, 300, 2048))


def test_gemm_wide_renorm(moe, orc):
    """d 4096 (16 raw chunks), d_ff 2048, top-2 renormalised, Q4_0"""
    L = orc.make_layer(34, 4096, 2048, 8, 2, orc.Q4_0, renorm=True)
    check_vs_oracle(moe, orc, L, orc.make_tokens(98, 150, 4096))


@pytest.mark.parametrize("T", [1024, 4096])
def test_gemm_matches_decode_kernels_at_large_batches(moe, orc, olmoe, T):
    """the decode kernels are fp32-accurate (checked against the oracle in
    the other tests); at large T they stand in for the oracle"""
    x = orc.make_tokens(99, T, 2048)
    lay = build(moe, olmoe)
    got = lay.forward(x)
    ref = lay.forward(x, flags=moe.FORCE_GEMV)
    assert np.isfinite(got).all()
    assert float(np.abs(got - ref).max()) <= TIGHT_ABS
    assert rel_l2(got, ref) <= TIGHT_REL
    lay.close()


def test_gemm_deterministic(moe, orc, q4_layer):
    x = orc.make_tokens(100, 200, 2048)
    lay = build(moe, q4_layer)
    a = lay.forward(x)
    b = lay.forward(x)
    np.testing.assert_array_equal(a, b)
    lay.close()
