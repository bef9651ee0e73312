"""GPU parity of the same-signature drop-ins and the dense quantized GEMV
against the CPU oracle."""
import numpy as np
import pytest

from test_gpu_moe import assert_output_close, rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qt", [1, 2])
@pytest.mark.parametrize("m", [1, 3])
def test_mma_transposed_quantized(moe, orc, qt, m):
    k, n = 512, 96
    w = orc.quantize(qt, orc.gauss(21, 7, n * k, 0.02).reshape(n, k))
    a = orc.gauss(21, 8, m * k, 1.0).reshape(m, k)
    ref = orc.gemm_q(a, w, qt, n)
    got = moe.mma_transposed(a, w, qt, n, k)
    assert rel_l2(got, ref) < 1e-5
    bias = orc.gauss(21, 9, n, 1.0)
    got_b = moe.mma_transposed(a, w, qt, n, k, add=bias)
    np.testing.assert_allclose(got_b, ref + bias, rtol=1e-5, atol=1e-5)


def test_mma_transposed_fp32_is_bit_exact(moe, orc):
    """fp32 rhs (the router GEMM) follows the 16-lane FMA chains exactly."""
    a = orc.gauss(5, 1, 7 * 2048, 1.0).reshape(7, 2048)
    wr = orc.gauss(5, 2, 64 * 2048, 0.02).reshape(64, 2048)
    got = moe.mma_transposed(a, wr, orc.F32, 64, 2048)
    np.testing.assert_array_equal(got, orc.router_logits(a, wr, 16))


def test_mma_transposed_fp32_odd_k_tail(moe, orc):
    a = orc.gauss(6, 1, 3 * 100, 1.0).reshape(3, 100)
    wr = orc.gauss(6, 2, 5 * 100, 0.5).reshape(5, 100)
    got = moe.mma_transposed(a, wr, orc.F32, 5, 100)
    np.testing.assert_array_equal(got, orc.router_logits(a, wr, 16))


@pytest.mark.parametrize("qt", [1, 2])
def test_fused_ffn_silu(moe, orc, qt):
    d, F = 512, 256
    g = orc.quantize(qt, orc.gauss(8, 2, F * d, 0.02).reshape(F, d))
    u = orc.quantize(qt, orc.gauss(8, 3, F * d, 0.02).reshape(F, d))
    dn = orc.quantize(qt, orc.gauss(8, 4, d * F, 0.02).reshape(d, F))
    x = orc.gauss(8, 5, d, 1.0)
    out, hidden, rc = moe.fused_ffn_silu(x, g, u, dn, qt, F)
    assert rc == 1
    lay = dict(router_w=np.zeros((1, d), np.float32), gate=g[None], up=u[None], down=dn[None],
               qtype=qt, d_model=d, d_ff=F, n_experts=1, top_k=1)
    ref, *_ = orc.moe_ffn(lay, x[None])
    assert_output_close(out[None], ref)


def test_fused_ffn_silu_not_applicable(moe, orc):
    """nn.c:503-507: two tokens -> 0, caller falls back."""
    d, F = 64, 32
    g = orc.quantize(1, np.zeros((F, d), np.float32))
    x = np.zeros((2, d), np.float32)
    import ctypes as C
    ts = [moe.tensor(x), moe.tensor(np.zeros((2, d), np.float32)),
          moe.tensor(np.zeros((1, F), np.float32)), moe.tensor(g, 1, (F, d)),
          moe.tensor(np.zeros((1, F), np.float32)), moe.tensor(g, 1, (F, d)),
          moe.tensor(orc.quantize(1, np.zeros((d, F), np.float32)), 1, (d, F))]
    assert moe.lib().moe_fused_ffn_silu(*[C.byref(t) for t in ts]) == 0


def test_config1_dense_q4_0_gemv(moe, orc):
    """W 14336x4096 Q4_0, x 1x4096, seed 1."""
    rows, cols = 14336, 4096
    w = orc.quantize(orc.Q4_0, orc.gauss(1, 7, rows * cols, 0.02).reshape(rows, cols))
    x = orc.gauss(1, 8, cols, 1.0)
    ref = orc.gemm_q(x[None], w, orc.Q4_0, rows)
    got = moe.gemv(w, orc.Q4_0, rows, cols, x)
    assert_output_close(got, ref)


def test_invalid_arguments_fail_cleanly(moe, orc):
    with pytest.raises(moe.MoeError):
        moe.gemv(np.zeros(34, np.uint8), orc.Q8_0, 1, 33, np.zeros(33, np.float32))
    with pytest.raises(moe.MoeError):
        moe.Layer(256, 128, 300, 4, 1, np.zeros((300, 256), np.float32),
                  np.zeros((300, 128, 272), np.uint8), np.zeros((300, 128, 272), np.uint8),
                  np.zeros((300, 256, 136), np.uint8))


@pytest.mark.parametrize("qt", [1, 2])
@pytest.mark.parametrize("rows,cols", [(100, 1024), (37, 2048), (8200, 1024)])
@pytest.mark.parametrize("m", [1, 5])
def test_gemv_partial_row_tiles(moe, orc, qt, rows, cols, m):
    """row counts that end inside a 16- or 32-row tile: the last tile's
    missing rows are neither computed into nor stored"""
    w = orc.quantize(qt, orc.gauss(41, 7, rows * cols, 0.02).reshape(rows, cols))
    x = orc.gauss(41, 8, m * cols, 1.0).reshape(m, cols)
    ref = orc.gemm_q(x, w, qt, rows)
    got = moe.gemv(w, qt, rows, cols, x)
    assert got.shape == ref.shape
    assert_output_close(got, ref)


@pytest.mark.parametrize("qt,rows,cols", [(1, 3, 64), (2, 5, 64), (1, 7, 192), (2, 1, 4160),
                                          (1, 33, 96), (2, 2, 128)])
def test_gemv_single_row(moe, orc, qt, rows, cols):
    """one activation row: the warp-per-row GEMV (rows of an even number of
    blocks; 96 columns = 3 blocks takes the general path) is fp32-accurate"""
    w = orc.quantize(qt, orc.gauss(43, 7, rows * cols, 0.02).reshape(rows, cols))
    x = orc.gauss(43, 8, cols, 1.0)
    ref = orc.gemm_q(x[None], w, qt, rows)
    got = moe.gemv(w, qt, rows, cols, x)
    assert got.shape == ref.shape
    assert float(np.abs(got - ref).max()) <= 1e-5
    assert rel_l2(got, ref) <= 1e-5


@pytest.mark.parametrize("qt,rows,cols", [(2, 37, 256), (1, 50, 512), (2, 16, 4096),
                                          (1, 100, 2304), (2, 33, 14336), (1, 17, 14336),
                                          (2, 2048, 4096), (1, 9, 16384), (2, 5, 16640)])
def test_gemv_single_row_large(moe, orc, qt, rows, cols):
    """one activation row at model sizes: rows of 256 to 16640 columns (one
    to four load rounds per lane, the 14336-column down projection among
    them), more rows than the grid has warps (2048), fp32-accurate"""
    w = orc.quantize(qt, orc.gauss(47, 7, rows * cols, 0.02).reshape(rows, cols))
    x = orc.gauss(47, 8, cols, 1.0)
    ref = orc.gemm_q(x[None], w, qt, rows)
    got = moe.gemv(w, qt, rows, cols, x)
    assert got.shape == ref.shape
    assert float(np.abs(got - ref).max()) <= 1e-5
    assert rel_l2(got, ref) <= 1e-5


@pytest.mark.parametrize("qt", [1, 2])
def test_gemv_single_row_unaligned_weights(moe, orc, qt):
    """weights 4 bytes past a 16-byte boundary (the kernel needs 4-byte
    alignment only: its loads are aligned 32-bit words)"""
    rows, cols = 40, 512
    w = orc.quantize(qt, orc.gauss(49, 7, rows * cols, 0.02).reshape(rows, cols))
    x = orc.gauss(49, 8, cols, 1.0)
    ref = orc.gemm_q(x[None], w, qt, rows)
    bw = moe.DeviceBuffer(w.nbytes + 16)
    bx = moe.DeviceBuffer.from_numpy(x)
    by = moe.DeviceBuffer(rows * 4)
    try:
        moe.check(moe.lib().moe_memcpy_h2d(bw.ptr + 4, np.ascontiguousarray(w).ctypes.data, w.nbytes))
        moe.gemv_device(bw.ptr + 4, qt, rows, cols, bx.ptr, 1, by.ptr)
        moe.check(moe.lib().moe_sync())
        got = by.to_numpy(np.float32, (1, rows))
    finally:
        for b in (bw, bx, by):
            b.free()
    assert float(np.abs(got - ref).max()) <= 1e-5
    assert rel_l2(got, ref) <= 1e-5


@pytest.mark.parametrize("qt,rows,cols,m", [(1, 2048, 2048, 512), (1, 384, 2048, 200),
                                             (2, 256, 14336, 80), (2, 640, 4096, 65),
                                             (1, 128, 1024, 300)])
def test_dense_gemm_prefill_sizes(moe, orc, qt, rows, cols, m):
    """more than 64 activation rows (prefill Q/K/V/O projections, lm_head):
    the tcgen05 GEMM with the matrix as one expert; rows that end in a
    128-row block (lm_head's 50304 = 393 x 128) are masked in the epilogue"""
    w = orc.quantize(qt, orc.gauss(51, 7, rows * cols, 0.02).reshape(rows, cols))
    x = orc.gauss(51, 8, m * cols, 1.0).reshape(m, cols)
    ref = orc.gemm_q(x, w, qt, rows)
    got = moe.gemv(w, qt, rows, cols, x)
    assert got.shape == ref.shape
    assert_output_close(got, ref)


def test_dense_gemm_drop_in_with_bias(moe, orc):
    """the tensor_mma_transposed_2x2 drop-in at prefill size (m = 96 > 64)"""
    m, n, k = 96, 256, 2048
    lhs = orc.gauss(52, 8, m * k, 1.0).reshape(m, k)
    rhs = orc.quantize(1, orc.gauss(52, 7, n * k, 0.02).reshape(n, k))
    add = orc.gauss(52, 9, n, 1.0)
    got = moe.mma_transposed(lhs, rhs, 1, n, k, add=add)
    ref = orc.gemm_q(lhs, rhs, 1, n) + add[None, :]
    assert_output_close(got, ref)
