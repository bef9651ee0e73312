"""The CPU oracle against the reference compiled from its own sources
(oracle/_ref, built by oracle/Makefile when the reference sources are present).
Bit-exact: both follow the reference's floating-point operation order.
Skipped where the compiled reference is absent."""
import numpy as np
import pytest


def need_ref(orc, variant):
    if not orc.ref_available(variant):
        pytest.skip(f"oracle/_ref/libref_{variant}.so not built")


VARIANTS = [("avx512", 16), ("avx2", 8)]


@pytest.mark.parametrize("variant,lanes", VARIANTS)
@pytest.mark.parametrize("qt", [1, 2])
@pytest.mark.parametrize("renorm", [0, 1])
def test_layer_bit_exact(orc, variant, lanes, qt, renorm):
    need_ref(orc, variant)
    L = orc.make_layer(7, 256, 128, 16, 4, qt, renorm=renorm, zipf=True)
    x = orc.make_tokens(7, 5, 256)
    out, ids, w, _ = orc.moe_ffn(L, x, lanes=lanes)
    r = orc.ref_call("moe", variant, x=x, router_w=L["router_w"], gate=L["gate"], up=L["up"],
                     down=L["down"], qtype=qt, d_ff=128, top_k=4, renorm=renorm,
                     router_bias=L["router_bias"])
    np.testing.assert_array_equal(ids, r["ids"])
    np.testing.assert_array_equal(w, r["w"])
    np.testing.assert_array_equal(out, r["out"])


def test_top_k_quirk_layer_bit_exact(orc):
    need_ref(orc, "avx512")
    L = orc.make_layer(8, 256, 128, 16, 4, orc.Q8_0)
    L["router_bias"] = np.zeros(16, np.float32)
    L["router_bias"][0] = 1.5
    x = orc.make_tokens(8, 12, 256)
    out, ids, w, _ = orc.moe_ffn(L, x)
    assert any((row == 0).sum() > 1 for row in ids)
    r = orc.ref_call("moe", "avx512", x=x, router_w=L["router_w"], gate=L["gate"], up=L["up"],
                     down=L["down"], qtype=1, d_ff=128, top_k=4, renorm=0,
                     router_bias=L["router_bias"])
    np.testing.assert_array_equal(ids, r["ids"])
    np.testing.assert_array_equal(out, r["out"])


@pytest.mark.parametrize("variant,lanes", VARIANTS)
@pytest.mark.parametrize("qt,m,k", [(1, 1, 512), (2, 1, 512), (1, 3, 512), (2, 3, 96)])
def test_gemm_bit_exact(orc, variant, lanes, qt, m, k):
    need_ref(orc, variant)
    a = orc.gauss(3, 9, m * k, 1.0).reshape(m, k)
    wq = orc.quantize(qt, orc.gauss(3, 10, 40 * k, 0.02).reshape(40, k))
    c = orc.gemm_q(a, wq, qt, 40, lanes)
    r = orc.ref_call("gemm", variant, a=a, b=wq, qtype=qt, n=40)
    np.testing.assert_array_equal(c, r["c"])


def test_quantize_softmax_topk_bit_exact(orc):
    need_ref(orc, "avx512")
    x = orc.gauss(1, 1, 8 * 64, 3.0).reshape(8, 64)
    np.testing.assert_array_equal(orc.quantize(orc.Q8_0, x), orc.ref_call("q8", x=x)["q"])
    np.testing.assert_array_equal(orc.softmax(x), orc.ref_call("softmax", v=x)["v"])
    ids = np.stack([orc.top_k(row, 8)[0] for row in x])
    np.testing.assert_array_equal(ids, orc.ref_call("topk", v=x, k=8)["ids"])


@pytest.mark.parametrize("qt", [1, 2])
def test_fused_ffn_bit_exact(orc, qt):
    need_ref(orc, "avx512")
    d, F = 512, 256
    g = orc.quantize(qt, orc.gauss(8, 2, F * d, 0.02).reshape(F, d))
    u = orc.quantize(qt, orc.gauss(8, 3, F * d, 0.02).reshape(F, d))
    dn = orc.quantize(qt, orc.gauss(8, 4, d * F, 0.02).reshape(d, F))
    x = orc.gauss(8, 5, d, 1.0)
    hidden = np.empty(F, np.float32)
    out = np.empty(d, np.float32)
    orc.lib().orc_fused_ffn_silu(x.ctypes.data, d, F, qt, g.ctypes.data, u.ctypes.data,
                                 dn.ctypes.data, 16, hidden.ctypes.data, out.ctypes.data)
    r = orc.ref_call("ffn", x=x, gate=g, up=u, down=dn, qtype=qt, d_ff=F)
    assert int(r["ok"]) == 1
    np.testing.assert_array_equal(out, r["out"])


# ---------------------------------------------------------------- K-quants
def test_q8K_quantizer_bit_exact(orc):
    """quant.c:627-654 (Q8_K activations), zeros and a first-of-ties maximum"""
    need_ref(orc, "avx512")
    rng = np.random.default_rng(11)
    x = rng.normal(0, 1, 1024).astype(np.float32)
    x[256:512] = 0.0                       # an all-zero block
    x[600], x[700] = 3.5, -3.5             # equal magnitudes: the first sets the sign
    r = orc.ref_call("q8k", "avx512", x=x)
    np.testing.assert_array_equal(orc.quantize_q8K(x), r["q"])


@pytest.mark.parametrize("qt", [3, 5])
def test_kquant_integer_dot_bit_exact(orc, qt):
    """quant_avx2.h: Q4_K / Q6_K rows against Q8_K activations"""
    need_ref(orc, "avx512")
    rng = np.random.default_rng(12 + qt)
    d = 2048
    x = rng.normal(0, 1, d).astype(np.float32)
    q8 = orc.quantize_q8K(x)
    w = orc.random_kquant(qt, rng, 24, d)
    mine = np.array([orc.dot_q8K(q8, w, qt, r, d) for r in range(24)], np.float32)
    ref = orc.ref_call("dotq8k", "avx512", q8=q8, q=w, qtype=qt, n=d, rows=24)["y"]
    np.testing.assert_array_equal(mine, ref)


@pytest.mark.parametrize("variant,lanes", VARIANTS)
@pytest.mark.parametrize("qt", [3, 5])
def test_kquant_f32_dot_bit_exact(orc, variant, lanes, qt):
    """quant.c:198-418: fp32 activations against Q4_K / Q6_K rows, lane order"""
    need_ref(orc, variant)
    rng = np.random.default_rng(13 + qt)
    d = 1024
    x = rng.normal(0, 1, d).astype(np.float32)
    w = orc.random_kquant(qt, rng, 16, d)
    mine = np.array([orc.dot_f32_quant(x, w, qt, r, d, lanes) for r in range(16)], np.float32)
    ref = orc.ref_call("dot", variant, x=x, q=w, qtype=qt, n=d, rows=16)["y"]
    np.testing.assert_array_equal(mine, ref)


@pytest.mark.parametrize("variant,lanes", VARIANTS)
@pytest.mark.parametrize("gu,dn", [(3, 5), (3, 3), (5, 5)])
def test_kquant_layer_bit_exact(orc, variant, lanes, gu, dn):
    """a MoE layer with K-quant experts: gate/up by the integer dots against
    Q8_K activations, down by the fp32 dot on h (nn.c:449-539, Q8_DOT)"""
    need_ref(orc, variant)
    L = orc.make_layer_kquant(14, 512, 256, 8, 2, gu, dn)
    x = orc.make_tokens(14, 5, 512)
    out, ids, w, _ = orc.moe_ffn(L, x, lanes=lanes)
    r = orc.ref_call("moe", variant, x=x, router_w=L["router_w"], gate=L["gate"], up=L["up"],
                     down=L["down"], qtype=L["qtype"], d_ff=256, top_k=2, renorm=0)
    np.testing.assert_array_equal(ids, r["ids"])
    np.testing.assert_array_equal(out, r["out"])
