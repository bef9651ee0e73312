"""The fused decode-layer kernel (one cooperative launch per layer forward)
against the CPU oracle and against the five-launch path.

Decode-sized batches (T <= 64) with d_model a multiple of 2048 take the
fused kernel; MOE_NO_FUSE forces the five-launch path.  Both run the same
expert pipeline over the same cost-balanced item partition and the same
lane-ordered router chains, so their outputs agree bit for bit.
"""
import numpy as np
import pytest

from test_gpu_moe import assert_dispatch, assert_output_close, assert_routing, build

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def olmoe(orc):
    """d 2048, 64 experts, top-8, d_ff 1024, Q8_0, seed 0."""
    return orc.make_layer(0, 2048, 1024, 64, 8, orc.Q8_0)


@pytest.fixture(scope="module")
def q4_layer(orc):
    """Q4_0 experts at a fused shape: d 2048, d_ff 1024, 16 experts, top-4."""
    return orc.make_layer(31, 2048, 1024, 16, 4, orc.Q4_0)


@pytest.fixture(scope="module")
def wide_layer(orc):
    """d 4096, d_ff 2048 (2048-column down stages), 8 experts top-2 renormalised,
    Q4_0: the Mixtral layer's structure at a smaller d_ff."""
    return orc.make_layer(32, 4096, 2048, 8, 2, orc.Q4_0, renorm=True)


def check(moe, orc, L, x, flags=0, lanes=16, mode=0):
    T = x.shape[0]
    ref, ids_ref, w_ref, _ = orc.moe_ffn(L, x, lanes=lanes, topk_mode=mode)
    lay = build(moe, L, flags=moe.RENORM if L.get("renorm") else 0)
    got = lay.forward(x, flags=flags | moe.NO_T1)
    ids, w, counts, offsets, perm = lay.routing(T)
    assert_routing(orc, x, L, lanes, ids, w, ids_ref, w_ref)
    assert_dispatch(orc, ids, counts, offsets, perm, L["n_experts"])
    assert_output_close(got, ref)
    five = lay.forward(x, flags=flags | moe.NO_FUSE)
    np.testing.assert_array_equal(got, five)
    lay.close()
    return got


@pytest.mark.parametrize("T", [1, 2, 7, 32, 64])
def test_fused_config0(moe, orc, olmoe, T):
    x = orc.make_tokens(0, 64, 2048)[:T]
    check(moe, orc, olmoe, x)


@pytest.mark.parametrize("T", [1, 9, 33])
def test_fused_q4_0(moe, orc, q4_layer, T):
    check(moe, orc, q4_layer, orc.make_tokens(40 + T, T, 2048))


@pytest.mark.parametrize("T", [1, 5, 64])
def test_fused_wide_renorm(moe, orc, wide_layer, T):
    check(moe, orc, wide_layer, orc.make_tokens(50 + T, T, 4096))


@pytest.mark.parametrize("flags,lanes,mode", [(1, 16, 1), (4, 8, 0), (5, 8, 1)])
def test_fused_modes(moe, orc, q4_layer, flags, lanes, mode):
    check(moe, orc, q4_layer, orc.make_tokens(60, 24, 2048), flags=flags, lanes=lanes,
          mode=mode)


def test_fused_zipf_and_quirk(moe, orc, q4_layer):
    L = dict(q4_layer)
    L["router_bias"] = orc.zipf_bias(4, 16, 1.1)
    check(moe, orc, L, orc.make_tokens(61, 48, 2048))
    # expert 0 dominant: the reference's top_k seeding repeats it in every slot
    bias = np.zeros(16, np.float32)
    bias[0] = 8.0
    L["router_bias"] = bias
    x = orc.make_tokens(62, 6, 2048)
    _, ids_ref, _, _ = orc.moe_ffn(L, x)
    assert (ids_ref == 0).all()
    check(moe, orc, L, x)


def test_fused_repeated_calls_and_batch_sizes(moe, orc, olmoe):
    """the grid barrier state carries over between launches of one layer,
    across batch sizes and after a five-launch forward"""
    lay = build(moe, olmoe)
    outs = {}
    for T in (3, 64, 1, 3, 17, 64):
        x = orc.make_tokens(70, 64, 2048)[:T]
        got = lay.forward(x)
        if T in outs:
            np.testing.assert_array_equal(got, outs[T])
        outs[T] = got
        lay.forward(x, flags=moe.NO_FUSE)
    ref, *_ = orc.moe_ffn(olmoe, orc.make_tokens(70, 64, 2048)[:17])
    assert_output_close(outs[17], ref)
    lay.close()


def test_fused_stage_times(moe, orc, olmoe):
    lay = build(moe, olmoe)
    x = orc.make_tokens(0, 32, 2048)
    lay.forward(x, flags=moe.PROFILE)
    lay.forward(x, flags=moe.PROFILE)
    ms, n = lay.stage_ms()
    assert n == 2
    assert all(v > 0 for v in ms), ms
    assert sum(ms) / n < 5.0, ms
    lay.close()


def test_beyond_fused_limit_takes_five_launch_path(moe, orc, olmoe):
    x = orc.make_tokens(80, 65, 2048)
    ref, ids_ref, w_ref, _ = orc.moe_ffn(olmoe, x)
    lay = build(moe, olmoe)
    got = lay.forward(x)
    ids, w, *_ = lay.routing(65)
    assert_routing(orc, x, olmoe, 16, ids, w, ids_ref, w_ref)
    assert_output_close(got, ref)
    lay.close()


@pytest.mark.parametrize("T", [1, 3, 5])
@pytest.mark.parametrize("flags,lanes,mode", [(0, 16, 0), (1, 16, 1), (4, 8, 0), (5, 8, 1)])
def test_fused_few_tokens_modes(moe, orc, q4_layer, T, flags, lanes, mode):
    """up to 8 tokens: one router expert per CTA; up to 5: the CTA-parallel
    top-k; up to 32 pairs: the one-warp dispatch (both lane orders, reference
    and exact top-k)"""
    check(moe, orc, q4_layer, orc.make_tokens(70 + T, T, 2048), flags=flags, lanes=lanes,
          mode=mode)


@pytest.mark.parametrize("bias0", [8.0, 1.5])
def test_fused_few_tokens_quirk(moe, orc, q4_layer, bias0):
    """the index-0 seeding quirk through the CTA-parallel top-k"""
    L = dict(q4_layer)
    bias = np.zeros(16, np.float32)
    bias[0] = bias0
    L["router_bias"] = bias
    check(moe, orc, L, orc.make_tokens(80, 4, 2048))
