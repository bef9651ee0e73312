"""MoE layers with K-quant experts (Q4_K / Q6_K, the formats of the
reference's real checkpoints) on the GPU (kquant.cu) against the oracle,
which is bit-exact against the reference compiled here
(tests/test_oracle_vs_ref.py): the gate/up integer dots against Q8_K
activations match the reference's operations; the down dot sums fp32 in a
warp's order instead of SIMD lanes, so outputs are checked at the layer
tolerance (max-abs 2e-3, rel-L2 1e-3) and expert ids exactly."""
import numpy as np
import pytest

from test_gpu_moe import assert_dispatch, assert_output_close, assert_routing, build

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("gu,dn", [(3, 5), (3, 3), (5, 5)])
@pytest.mark.parametrize("T", [1, 3, 17, 100])
def test_kquant_layer(moe, orc, gu, dn, T):
    L = orc.make_layer_kquant(40 + gu + dn, 512, 256, 8, 2, gu, dn)
    x = orc.make_tokens(41 + T, T, 512)
    ref, ids_ref, w_ref, _ = orc.moe_ffn(L, x)
    lay = build(moe, L)
    got = lay.forward(x)
    ids, w, counts, offsets, perm = lay.routing(T)
    assert_routing(orc, x, L, 16, ids, w, ids_ref, w_ref)
    assert_dispatch(orc, ids, counts, offsets, perm, 8)
    assert_output_close(got, ref)
    lay.close()


def test_kquant_olmoe_shape_decode(moe, orc):
    """the OLMoE layer shape (d 2048, 64 experts top-8, d_ff 1024) in
    Q4_K_M's types, one decode token and a short batch"""
    L = orc.make_layer_kquant(50, 2048, 1024, 64, 8, orc.Q4_K, orc.Q6_K)
    lay = build(moe, L)
    for T in (1, 6):
        x = orc.make_tokens(51 + T, T, 2048)
        ref, ids_ref, w_ref, _ = orc.moe_ffn(L, x)
        got = lay.forward(x)
        ids, w, *_ = lay.routing(T)
        assert_routing(orc, x, L, 16, ids, w, ids_ref, w_ref)
        assert_output_close(got, ref)
    lay.close()


def test_kquant_tensor_t_dropin(moe, orc):
    """moe_ffn_forward with tensor_t views of K-quant 3-D expert tensors
    (gate/up Q4_K, down Q6_K, as olmoe.c passes them for a Q4_K_M file)"""
    L = orc.make_layer_kquant(60, 512, 256, 8, 2, orc.Q4_K, orc.Q6_K)
    x = orc.make_tokens(61, 4, 512)
    ref, *_ = orc.moe_ffn(L, x)
    got = moe.ffn_forward(x, L["router_w"], L["gate"], L["up"], L["down"],
                          moe.qtype2(moe.Q4_K, moe.Q6_K), 2)
    assert_output_close(got, ref)


def test_kquant_rejects_unsupported(moe, orc):
    L = orc.make_layer_kquant(70, 512, 256, 8, 2, orc.Q4_K, orc.Q6_K)
    L = dict(L, qtype=moe.qtype2(moe.Q4_K, moe.Q8_0))   # mixed legacy / K-quant
    with pytest.raises(moe.MoeError):
        build(moe, L)
