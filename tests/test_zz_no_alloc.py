"""moe_gemv_device_noalloc, collected last (the file name sorts after every
other test module).

This entry point is for callers that cannot allocate device memory where they
call the GEMV: a real-time decode loop that must not take cudaMalloc's
implicit synchronisation, or an engine whose device memory budget is fixed and
handed out by someone else.  Its scratch lives in a fixed 1 MiB device array
inside the library (the previous call's contents stay in it), so it must give
the same results as the allocating moe_gemv_device, call after call.
"""
import numpy as np
import pytest

from test_gpu_moe import MAX_ABS, REL_L2, rel_l2

pytestmark = pytest.mark.gpu

CASES = [
    (1, 4096, 2048, 1),   # Q8_0, tensor-core path
    (2, 2048, 4096, 3),   # Q4_0, tensor-core path
    (1, 96, 96, 2),       # Q8_0, cols not a multiple of 256: CUDA-core path
]


@pytest.mark.parametrize("qt,rows,cols,m", CASES)
def test_noalloc_matches_allocating_gemv_twice(moe, orc, qt, rows, cols, m):
    w = orc.quantize(qt, orc.gauss(31, 7, rows * cols, 0.02).reshape(rows, cols))
    dw = moe.DeviceBuffer.from_numpy(w)
    dy_ref = moe.DeviceBuffer(m * rows * 4)
    dy = moe.DeviceBuffer(m * rows * 4)
    for call in range(2):
        x = orc.gauss(32 + call, 8, m * cols, 1.0).reshape(m, cols)
        dx = moe.DeviceBuffer.from_numpy(x)
        moe.gemv_device(dw.ptr, qt, rows, cols, dx.ptr, m, dy_ref.ptr)
        moe.check(moe.lib().moe_gemv_device_noalloc(dw.ptr, qt, rows, cols, dx.ptr, m, dy.ptr,
                                                     None))
        moe.check(moe.lib().moe_sync())
        ref = dy_ref.to_numpy(np.float32, (m, rows))
        got = dy.to_numpy(np.float32, (m, rows))
        assert np.isfinite(got).all()
        assert float(np.abs(got - ref).max()) <= MAX_ABS
        assert rel_l2(got, ref) <= REL_L2
        # and against the CPU oracle of the reference's dot products
        assert rel_l2(got, orc.gemm_q(x, w, qt, rows)) <= REL_L2


def test_noalloc_rejects_sizes_beyond_its_scratch(moe, orc):
    rows, cols, m = 8, 8192, 64          # m * cols = 524288 > 262080
    dw = moe.DeviceBuffer(rows * cols // 32 * 34)
    dx = moe.DeviceBuffer(m * cols * 4)
    dy = moe.DeviceBuffer(m * rows * 4)
    rc = moe.lib().moe_gemv_device_noalloc(dw.ptr, 1, rows, cols, dx.ptr, m, dy.ptr, None)
    assert rc == -1
    assert b"exceeds the fixed scratch" in moe.lib().moe_last_error()
