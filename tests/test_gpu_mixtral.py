"""The MoE layer at the Mixtral-8x7B shape (d_model 4096, d_ff 14336, 8
experts, top-2 with the softmax renormalised over the selected pair, Q4_0
experts: 99 MB per expert) against the CPU oracle, through both paths: the
fused decode kernel for a few tokens and the grouped tcgen05 GEMM.  The layer
is the one config 3 runs in every one of its 32 layers."""
import numpy as np
import pytest

from test_gpu_moe import assert_dispatch, assert_output_close, assert_routing, build, rel_l2

pytestmark = pytest.mark.gpu

D, F, NE, K = 4096, 14336, 8, 2


@pytest.fixture(scope="module")
def mixtral(orc):
    return orc.make_layer(3, D, F, NE, K, orc.Q4_0, renorm=True)


@pytest.fixture
def mixtral_layer(moe, mixtral):
    lay = build(moe, mixtral, flags=moe.RENORM)
    yield lay
    lay.close()


@pytest.mark.parametrize("T,path", [(3, "fused"), (24, "gemm")])
def test_mixtral_layer_matches_oracle(moe, orc, mixtral, mixtral_layer, T, path):
    x = orc.make_tokens(300 + T, T, D)
    ref, ids_ref, w_ref, _ = orc.moe_ffn(mixtral, x)
    got = mixtral_layer.forward(x, flags=moe.FORCE_GEMM if path == "gemm" else 0)
    ids, w, counts, offsets, perm = mixtral_layer.routing(T)
    assert_routing(orc, x, mixtral, 16, ids, w, ids_ref, w_ref)
    assert_dispatch(orc, ids, counts, offsets, perm, NE)
    assert_output_close(got, ref)
    # outputs reach |y| ~ 10 here: the decode kernels are fp32-accurate, the
    # GEMM carries its tensor-core accumulation (~7e-5 rel-L2)
    if path == "fused":
        assert float(np.abs(got - ref).max()) <= 1e-4
    assert rel_l2(got, ref) <= 1e-4


def test_mixtral_gemm_matches_decode_kernels_at_prefill(moe, orc, mixtral_layer):
    """256 tokens: the GEMM against the decode expert kernels, which are
    fp32-accurate (~1e-6, checked against the oracle above).  What separates
    them is the tensor cores' fp32 accumulation in the GEMM, which truncates:
    over K = 14336 it reaches ~7e-5 rel-L2 and ~9e-4 max-abs at |y| ~ 10,
    inside the north-star bar (2e-3 / 1e-3)."""
    x = orc.make_tokens(333, 256, D)
    got = mixtral_layer.forward(x)
    ref = mixtral_layer.forward(x, flags=moe.FORCE_GEMV)
    assert np.isfinite(got).all()
    assert float(np.abs(got - ref).max()) <= 1.5e-3
    assert rel_l2(got, ref) <= 1e-4
