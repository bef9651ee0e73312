"""The device generator and quantizer that build the benchmarked layers
(moe_synth_gauss, moe_quantize_device) against the CPU oracle's generator
and the reference quantizers' rounding rules (quant.c:62-78 for Q8_0,
test/quant.c:45-79 for Q4_0), so the layers bench.py measures are the
layers the oracle checks.

Both generators evaluate Box-Muller in double precision and round once to
fp32.  CUDA's double log/cos and glibc's may differ in the last bit of the
double, which changes the fp32 result only when the double lies within
~2^-29 of an fp32 rounding midpoint: about one value in 10^8-10^9.  So the
values must agree bit for bit except for at most one in a million, and then
by one ulp; given the same fp32 input, the quantizers must agree exactly.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def assert_same_values(got, ref):
    bad = np.flatnonzero(got.view(np.int32) != ref.view(np.int32))
    assert bad.size <= max(1, got.size // 1_000_000), bad.size
    if bad.size:
        ulps = np.abs(got[bad].view(np.int32).astype(np.int64) - ref[bad].view(np.int32))
        assert int(ulps.max()) <= 1


@pytest.mark.parametrize("seed,tag,offset,n,sd", [
    (0, 1, 0, 64 * 2048, 0.02),        # config-0 router weights
    (0, 5, 0, 32 * 2048, 1.0),         # config-0 tokens
    (0, 2, 5 * 1024 * 2048, 4 * 1024 * 2048, 0.02),  # experts 5-8 of config-0 gate
    (1, 2, 0, 1 << 20, 0.02),          # config-1 weights (prefix)
    (7, 4, 123, 1000, 0.5),            # odd offset and length
])
def test_synth_gauss_matches_oracle(moe, orc, seed, tag, offset, n, sd):
    buf = moe.DeviceBuffer(n * 4)
    moe.check(moe.lib().moe_synth_gauss(buf.ptr, seed, tag, offset, n, sd, None))
    moe.check(moe.lib().moe_sync())
    got = buf.to_numpy(np.float32, (n,))
    ref = orc.gauss(seed, tag, n, sd, offset=offset)
    assert_same_values(got, ref)


@pytest.mark.parametrize("qt,rows,cols", [(1, 1024, 2048), (2, 1024, 2048), (1, 64, 1024),
                                          (2, 256, 4096), (1, 3, 96)])
def test_quantize_device_matches_oracle(moe, orc, qt, rows, cols):
    x = orc.gauss(3, 2, rows * cols, 0.02).reshape(rows, cols)
    x[0, :32] = 0.0          # an all-zero block (scale 0)
    x[-1, -32:] *= 50.0      # a block with large values
    dx = moe.DeviceBuffer.from_numpy(x)
    dq = moe.DeviceBuffer(rows * moe.row_bytes(qt, cols))
    moe.check(moe.lib().moe_quantize_device(dx.ptr, rows, cols, qt, dq.ptr, None))
    moe.check(moe.lib().moe_sync())
    got = dq.to_numpy(np.uint8, (rows, moe.row_bytes(qt, cols)))
    ref = orc.quantize(qt, x).reshape(rows, -1)
    bad = np.argwhere(got != ref)
    assert bad.size == 0, [(tuple(i), int(got[tuple(i)]), int(ref[tuple(i)])) for i in bad[:8]]


def test_bench_layer_bytes_match_oracle_layer(moe, orc):
    """the first experts of a config-0 layer as bench.py generates them on the
    device (seed, tags 1-4, quantized on the device) are orc.make_layer's:
    the device quantizer applied to the device values equals the oracle's
    quantizer applied to them, and those values are the oracle's"""
    d, F, n = 2048, 1024, 2
    for tag, rows, cols in ((2, F, d), (3, F, d), (4, d, F)):
        tmp = moe.DeviceBuffer(n * rows * cols * 4)
        q = moe.DeviceBuffer(n * rows * moe.row_bytes(1, cols))
        moe.check(moe.lib().moe_synth_gauss(tmp.ptr, 0, tag, 0, n * rows * cols, 0.02, None))
        moe.check(moe.lib().moe_quantize_device(tmp.ptr, n * rows, cols, 1, q.ptr, None))
        moe.check(moe.lib().moe_sync())
        vals = tmp.to_numpy(np.float32, (n * rows, cols))
        got = q.to_numpy(np.uint8, (n * rows * moe.row_bytes(1, cols),))
        np.testing.assert_array_equal(got, orc.quantize(1, vals).reshape(-1))
        assert_same_values(vals.reshape(-1), orc.gauss(0, tag, n * rows * cols, 0.02))
