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


def test_noalloc_at_the_exact_size_limit_and_one_step_past(moe, orc):
    """m * cols == 262080 fits the scratch exactly; the next size up is refused"""
    qt, rows, m, cols = 1, 64, 15, 17472            # 15 * 17472 = 262080
    w = orc.quantize(qt, orc.gauss(33, 7, rows * cols, 0.02).reshape(rows, cols))
    x = orc.gauss(34, 8, m * cols, 1.0).reshape(m, cols)
    dw, dx = moe.DeviceBuffer.from_numpy(w), moe.DeviceBuffer.from_numpy(x)
    dy, dy_ref = moe.DeviceBuffer(m * rows * 4), moe.DeviceBuffer(m * rows * 4)
    moe.check(moe.lib().moe_gemv_device_noalloc(dw.ptr, qt, rows, cols, dx.ptr, m, dy.ptr, None))
    moe.gemv_device(dw.ptr, qt, rows, cols, dx.ptr, m, dy_ref.ptr)
    moe.check(moe.lib().moe_sync())
    got, ref = dy.to_numpy(np.float32, (m, rows)), dy_ref.to_numpy(np.float32, (m, rows))
    assert float(np.abs(got - ref).max()) <= MAX_ABS and rel_l2(got, ref) <= REL_L2
    dx2 = moe.DeviceBuffer((m + 1) * cols * 4)
    dy2 = moe.DeviceBuffer((m + 1) * rows * 4)
    rc = moe.lib().moe_gemv_device_noalloc(dw.ptr, qt, rows, cols, dx2.ptr, m + 1, dy2.ptr, None)
    assert rc == -1
    assert b"exceeds the fixed scratch" in moe.lib().moe_last_error()


def test_noalloc_on_a_caller_stream(moe, orc):
    """the real-time caller's case: its own stream, synchronised by itself"""
    import torch
    qt, rows, cols, m = 2, 1024, 4096, 2
    w = orc.quantize(qt, orc.gauss(35, 7, rows * cols, 0.02).reshape(rows, cols))
    dw = moe.DeviceBuffer.from_numpy(w)
    st = torch.cuda.Stream()
    for call in range(2):
        x = orc.gauss(36 + call, 8, m * cols, 1.0).reshape(m, cols)
        dx, dy = moe.DeviceBuffer.from_numpy(x), moe.DeviceBuffer(m * rows * 4)
        moe.check(moe.lib().moe_gemv_device_noalloc(dw.ptr, qt, rows, cols, dx.ptr, m, dy.ptr,
                                                     st.cuda_stream))
        st.synchronize()
        got = dy.to_numpy(np.float32, (m, rows))
        assert rel_l2(got, orc.gemm_q(x, w, qt, rows)) <= REL_L2


FRESH = r"""
import ctypes as C, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from conftest import load_package
from oracle import oracle as orc
moe = load_package()
L = moe.lib()
qt, rows, cols, m = 1, 512, 2048, 1
w = orc.quantize(qt, orc.gauss(37, 7, rows * cols, 0.02).reshape(rows, cols))
x = orc.gauss(38, 8, m * cols, 1.0).reshape(m, cols)
# device buffers through the CUDA runtime directly: the library is not
# initialised before the no-allocation call
rt = C.CDLL("libcudart.so.12")
def dalloc(n):
    p = C.c_void_p()
    assert rt.cudaMalloc(C.byref(p), C.c_size_t(n)) == 0
    return p.value
dw, dx, dy = dalloc(w.nbytes), dalloc(x.nbytes), dalloc(m * rows * 4)
assert rt.cudaMemcpy(C.c_void_p(dw), w.ctypes.data_as(C.c_void_p), C.c_size_t(w.nbytes), 1) == 0
assert rt.cudaMemcpy(C.c_void_p(dx), x.ctypes.data_as(C.c_void_p), C.c_size_t(x.nbytes), 1) == 0
rc = L.moe_gemv_device_noalloc(dw, qt, rows, cols, dx, m, dy, None)
assert rc == 0, (rc, L.moe_last_error())
assert L.moe_sync() == 0, L.moe_last_error()
y = np.empty((m, rows), np.float32)
assert rt.cudaMemcpy(y.ctypes.data_as(C.c_void_p), C.c_void_p(dy), C.c_size_t(y.nbytes), 2) == 0
err = float(np.linalg.norm(y - orc.gemm_q(x, w, qt, rows)) / np.linalg.norm(y))
print("REL", err)
"""


def test_noalloc_as_the_first_call_of_a_fresh_process(orc):
    """no moe_init, no other library call before it: a NULL stream makes the
    call initialise the library (a stream, no memory) on the current device"""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    out = subprocess.run([sys.executable, "-c", FRESH, here], capture_output=True, text=True, timeout=300,
                         cwd=os.path.dirname(here))
    assert out.returncode == 0, out.stderr[-2000:]
    rel = float(out.stdout.split("REL")[-1])
    assert rel <= REL_L2


def test_noalloc_rejects_sizes_beyond_its_scratch(moe, orc):
    rows, cols, m = 8, 8192, 64          # m * cols = 524288 > 262080
    dw = moe.DeviceBuffer(rows * cols // 32 * 34)
    dx = moe.DeviceBuffer(m * cols * 4)
    dy = moe.DeviceBuffer(m * rows * 4)
    rc = moe.lib().moe_gemv_device_noalloc(dw.ptr, 1, rows, cols, dx.ptr, m, dy.ptr, None)
    assert rc == -1
    assert b"exceeds the fixed scratch" in moe.lib().moe_last_error()
