"""Python binding of libmoe_b200.so (the B200 MoE FFN C ABI, include/moe_b200.h).

The product is the C ABI; this module is the thin ctypes mirror that the
tests and bench.py use.  It never computes anything itself and never falls
back to the CPU: if the shared library is missing it raises.

The directory name (llm.c_b200) is not a valid Python identifier, so load
it with `load_package()` from bench.py / tests/conftest.py, or by path.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmoe_b200.so")

F32, Q8_0, Q4_0, Q4_K, Q6_K = 0, 1, 2, 3, 5


def qtype2(gate_up: int, down: int) -> int:
    """MOE_QTYPE2: a layer's gate/up and down weight types"""
    return gate_up | (down << 8)
TOPK_EXACT, DEVICE_IO, LANES_AVX2, RENORM, FORCE_GEMV, FORCE_GEMM, PROFILE, SIMPLE = (
    0x1, 0x2, 0x4, 0x8, 0x10, 0x20, 0x40, 0x80)
NO_FUSE = 0x100
EP_SHARDED = 0x200
NO_T1 = 0x400
FORCE_T1 = 0x800

ERRORS = {0: "MOE_OK", -1: "MOE_ERR_INVALID", -2: "MOE_ERR_UNSUPPORTED", -3: "MOE_ERR_CUDA",
          -4: "MOE_ERR_NOMEM", -5: "MOE_ERR_NOT_INIT", -6: "MOE_ERR_COMM", -7: "MOE_ERR_TIMEOUT"}


class MoeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class MoeTensor(C.Structure):
    """Layout of the reference's tensor_t (tensor.h:19-31, -DQ8_DOT build)."""
    _fields_ = [("data", C.c_void_p), ("qdata", C.c_void_p), ("type", C.c_int),
                ("totlen", C.c_uint64), ("maxcap", C.c_uint64), ("dim", C.c_uint64 * 4),
                ("ndim", C.c_uint32), ("scratch", C.c_void_p), ("scratch_size", C.c_size_t)]


class LayerDesc(C.Structure):
    _fields_ = [("d_model", C.c_int64), ("d_ff", C.c_int64), ("n_experts", C.c_int64),
                ("top_k", C.c_int64), ("qtype", C.c_int), ("flags", C.c_int),
                ("router_w", C.c_void_p), ("router_bias", C.c_void_p),
                ("gate", C.POINTER(C.c_void_p)), ("up", C.POINTER(C.c_void_p)),
                ("down", C.POINTER(C.c_void_p)),
                ("first_expert", C.c_int64), ("n_local", C.c_int64)]


_TPP = C.POINTER(C.POINTER(MoeTensor))


class ModelDesc(C.Structure):
    """moe_model_desc (include/moe_b200.h)"""
    _fields_ = [("arch", C.c_int), ("n_layers", C.c_int64), ("d_model", C.c_int64),
                ("n_heads", C.c_int64), ("n_kv_heads", C.c_int64), ("head_len", C.c_int64),
                ("vocab", C.c_int64), ("context", C.c_int64), ("n_experts", C.c_int64),
                ("top_k", C.c_int64), ("d_ff", C.c_int64), ("rope_theta", C.c_float),
                ("token_embd", C.POINTER(MoeTensor)), ("output", C.POINTER(MoeTensor)),
                ("output_norm", C.POINTER(MoeTensor)),
                ("attn_norm", _TPP), ("attn_q", _TPP), ("attn_k", _TPP), ("attn_v", _TPP),
                ("attn_q_norm", _TPP), ("attn_k_norm", _TPP), ("attn_output", _TPP),
                ("ffn_norm", _TPP), ("ffn_gate_inp", _TPP),
                ("ffn_gate", _TPP), ("ffn_up", _TPP), ("ffn_down", _TPP)]


ARCH_OLMOE, ARCH_LLAMA = 0, 1

_lib = None

# every symbol include/moe_b200.h declares, with (restype, argtypes)
_P, _I, _SZ, _I64, _U64, _F = C.c_void_p, C.c_int, C.c_size_t, C.c_int64, C.c_uint64, C.c_float
_TP = C.POINTER(MoeTensor)
SIGNATURES = {
    "moe_init": (_I, [_I]),
    "moe_shutdown": (_I, []),
    "moe_last_error": (C.c_char_p, []),
    "moe_version": (C.c_char_p, []),
    "moe_register_weights": (_I, [_TP]),
    "moe_unregister_weights": (_I, [_TP]),
    "moe_resident_bytes": (_SZ, []),
    "moe_tensor_mma_transposed_2x2": (None, [_TP, _TP, _TP, _TP]),
    "moe_tensor_mma_transposed_2x2_status": (_I, [_TP, _TP, _TP, _TP]),
    "moe_fused_ffn_silu": (_I, [_TP, _TP, _TP, _TP, _TP, _TP, _TP]),
    "moe_ffn_forward": (_I, [_TP, _TP, _TP, _TP, _TP, _TP, _SZ, _I]),
    "moe_ffn_forward_split": (_I, [_TP, _TP, _TP, C.POINTER(_TP), C.POINTER(_TP),
                                   C.POINTER(_TP), _SZ, _SZ, _I]),
    "moe_layer_create": (_I, [C.POINTER(_P), C.POINTER(LayerDesc)]),
    "moe_layer_destroy": (_I, [_P]),
    "moe_layer_forward": (_I, [_P, _P, _P, _I64, _I, _P]),
    "moe_layer_routing": (_I, [_P, _P, _P, _P, _P, _P]),
    "moe_layer_status": (_I, [_P]),
    "moe_layer_set_wait_ms": (_I, [_P, _I]),
    "moe_layer_ep_reset": (_I, [_P]),
    "moe_layer_stage_ms": (_I, [_P, C.POINTER(C.c_float), _I]),
    "moe_layer_phase_stamps": (_I, [_P, C.POINTER(C.c_uint64), _I]),
    "moe_layer_ipc_handle": (_I, [_P, _P]),
    "moe_layer_set_peers": (_I, [_P, _I, _I, _P]),
    "moe_ep_unique_id": (_I, [_P]),
    "moe_ep_init": (_I, [_I, _I, _P]),
    "moe_ep_finalize": (_I, []),
    "moe_gemv_device": (_I, [_P, _I, _I64, _I64, _P, _I64, _P, _P]),
    "moe_gemv_device_noalloc": (_I, [_P, _I, _I64, _I64, _P, _I64, _P, _P]),
    "moe_sync": (_I, []),
    "moe_device_alloc": (_P, [_SZ]),
    "moe_device_free": (_I, [_P]),
    "moe_memcpy_h2d": (_I, [_P, _P, _SZ]),
    "moe_memcpy_d2h": (_I, [_P, _P, _SZ]),
    "moe_host_alloc": (_P, [_SZ]),
    "moe_host_free": (_I, [_P]),
    "moe_synth_gauss": (_I, [_P, _U64, _U64, _U64, _I64, _F, _P]),
    "moe_quantize_device": (_I, [_P, _I64, _I64, _I, _P, _P]),
    "moe_model_create": (_I, [C.POINTER(_P), C.POINTER(ModelDesc)]),
    "moe_model_destroy": (_I, [_P]),
    "moe_model_prefill": (_I, [_P, _P, _P, _SZ, _P]),
    "moe_model_decode": (_I, [_P, _I, _I, _P]),
    "moe_model_logits": (_I, [_P, _SZ, _P]),
    "moe_model_generate": (_I, [_P, _P, _SZ, _I, _I, _P]),
    "moe_model_reset": (_I, [_P]),
    "moe_model_timing": (_I, [_P, C.POINTER(C.c_float), C.POINTER(C.c_float)]),
    "moe_model_status": (_I, [_P]),
    "moe_model_mode": (_I, [_P]),
    "moe_model_info": (_I, [_P, C.POINTER(_I64), C.POINTER(_I64), C.POINTER(_SZ)]),
}


def lib():
    """Load libmoe_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `make -C llm.c_b200` "
                              "(or __graft_entry__.build()); there is no CPU fallback")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int):
    if rc != 0:
        raise MoeError(rc, lib().moe_last_error().decode())
    return rc


def init(device: int = 0):
    check(lib().moe_init(device))


def shutdown():
    check(lib().moe_shutdown())


def reset(device: int = 0):
    """Drop every registered weight and cached layer (moe_shutdown), then
    re-initialise.  Host-pointer-keyed registrations must not outlive the
    host buffers they mirror."""
    shutdown()
    init(device)


# ------------------------------------------------------------------ tensors
def row_bytes(qtype: int, cols: int) -> int:
    return {Q8_0: cols // 32 * 34, Q4_0: cols // 32 * 18, Q4_K: cols // 256 * 144,
            Q6_K: cols // 256 * 210, F32: cols * 4}[qtype]


def tensor_at(ptr: int, qtype: int, dims) -> MoeTensor:
    """tensor_t view of a raw (host or device) pointer"""
    t = MoeTensor()
    if qtype == F32:
        t.data = ptr
    else:
        t.qdata = ptr
    t.type = qtype
    t.ndim = len(dims)
    n = 1
    for i, dd in enumerate(dims):
        t.dim[i] = dd
        n *= dd
    t.totlen = n
    t.maxcap = n
    return t


def tensor(arr: np.ndarray, qtype: int = F32, dims=None) -> MoeTensor:
    """tensor_t view of a numpy array: fp32 data, or uint8 GGUF blocks with
    logical dims (outermost first, innermost = columns)."""
    t = MoeTensor()
    if qtype == F32:
        dims = arr.shape if dims is None else dims
        t.data = arr.ctypes.data
    else:
        assert dims is not None
        t.qdata = arr.ctypes.data
    t.type = qtype
    t.ndim = len(dims)
    n = 1
    for i, dd in enumerate(dims):
        t.dim[i] = dd
        n *= dd
    t.totlen = n
    t.maxcap = n
    t._keep = arr
    return t


# ------------------------------------------------------------------ device memory
class DeviceBuffer:
    def __init__(self, nbytes: int):
        self.nbytes = nbytes
        self.ptr = lib().moe_device_alloc(max(nbytes, 1))
        if not self.ptr:
            raise MoeError(-4, lib().moe_last_error().decode())

    @classmethod
    def from_numpy(cls, a: np.ndarray) -> "DeviceBuffer":
        a = np.ascontiguousarray(a)
        b = cls(a.nbytes)
        if a.nbytes:
            check(lib().moe_memcpy_h2d(b.ptr, a.ctypes.data, a.nbytes))
        return b

    def to_numpy(self, dtype, shape) -> np.ndarray:
        out = np.empty(shape, dtype)
        if out.nbytes:
            check(lib().moe_memcpy_d2h(out.ctypes.data, self.ptr, out.nbytes))
        return out

    def free(self):
        if self.ptr:
            lib().moe_device_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


# ------------------------------------------------------------------ expert parallelism
def expert_range(rank: int, world: int, n_experts: int):
    """(first_expert, n_local) of `rank`: contiguous, balanced ranges that
    cover every expert once"""
    if world < 1 or not 0 <= rank < world or n_experts < world:
        raise ValueError(f"rank {rank} of {world} over {n_experts} experts")
    first = rank * n_experts // world
    return first, (rank + 1) * n_experts // world - first


def connect_expert_parallel(layer: "Layer", rank: int, all_gather) -> None:
    """exchange the layer's buffer handles between the ranks and connect them;
    `all_gather(obj) -> list` gathers one picklable object from every rank
    in rank order (e.g. torch.distributed.all_gather_object)"""
    layer.set_peers(rank, all_gather(layer.ipc_handle()))


def init_expert_parallel_comm(rank: int, world: int, all_gather) -> None:
    """create the library's NCCL communicator (moe_ep_init), once per process;
    rank 0's unique id travels through `all_gather` (as above)"""
    uid = (C.c_char * 128)()
    if rank == 0:
        check(lib().moe_ep_unique_id(uid))
    ids = all_gather(bytes(uid) if rank == 0 else None)
    buf = (C.c_char * 128).from_buffer_copy(ids[0])
    check(lib().moe_ep_init(rank, world, buf))


# ------------------------------------------------------------------ layer
class Layer:
    """Device-resident MoE layer (moe_layer_create).  `gate`/`up` are uint8
    [NE, d_ff, rb] and `down` uint8 [NE, d, rb] GGUF blocks, or device
    pointer lists when built from device data."""

    def __init__(self, d_model, d_ff, n_experts, top_k, qtype, router_w, gate, up, down,
                 router_bias=None, flags=0, first_expert=0, n_local=0):
        self.bufs = []
        self.d_model, self.d_ff, self.n_experts, self.top_k = d_model, d_ff, n_experts, top_k
        self.first_expert = first_expert
        self.n_local = n_local if n_local else n_experts - first_expert

        def dev(a):
            if isinstance(a, int):
                return a
            b = DeviceBuffer.from_numpy(a)
            self.bufs.append(b)
            return b.ptr

        f32 = lambda a: a if isinstance(a, int) else np.ascontiguousarray(a, np.float32)  # noqa: E731
        self.router_w = dev(f32(router_w))
        self.router_bias = None if router_bias is None else dev(f32(router_bias))

        def ptrs(m):
            if isinstance(m, (list, tuple)):
                return [int(p) for p in m]
            base = dev(np.ascontiguousarray(m))
            stride = m[0].nbytes
            return [base + e * stride for e in range(n_experts)]

        self._g = (C.c_void_p * n_experts)(*ptrs(gate))
        self._u = (C.c_void_p * n_experts)(*ptrs(up))
        self._d = (C.c_void_p * n_experts)(*ptrs(down))
        desc = LayerDesc(d_model, d_ff, n_experts, top_k, qtype, flags, self.router_w,
                         self.router_bias, C.cast(self._g, C.POINTER(C.c_void_p)),
                         C.cast(self._u, C.POINTER(C.c_void_p)),
                         C.cast(self._d, C.POINTER(C.c_void_p)), first_expert, n_local)
        h = C.c_void_p()
        check(lib().moe_layer_create(C.byref(h), C.byref(desc)))
        self.handle = h.value

    def forward_device(self, x_ptr: int, out_ptr: int, T: int, flags=0, stream=None):
        check(lib().moe_layer_forward(self.handle, x_ptr, out_ptr, T, flags, stream))

    def forward(self, x: np.ndarray, flags=0) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        bx = DeviceBuffer.from_numpy(x)
        bo = DeviceBuffer(x.nbytes)
        self.forward_device(bx.ptr, bo.ptr, T, flags)
        check(lib().moe_layer_status(self.handle))   # waits; raises on a device-side failure
        self.last_T = T
        return bo.to_numpy(np.float32, x.shape)

    def stage_ms(self):
        """(per-stage ms summed over profiled forwards, number of forwards)"""
        ms = (C.c_float * 6)()
        check(lib().moe_layer_stage_ms(self.handle, ms, 6))
        return list(ms)[:5], int(ms[5])

    PHASE_STAMPS = ("start", "router", "barrier1", "topk", "barrier1b", "dispatch", "routing",
                    "gate_up", "barrier2", "down", "barrier3", "end")

    def phase_stamps(self, n_ctas: int = 1024) -> np.ndarray:
        """raw %globaltimer stamps [CTA, 12] (ns) of the latest profiled fused forward"""
        buf = (C.c_uint64 * (n_ctas * len(self.PHASE_STAMPS)))()
        n = lib().moe_layer_phase_stamps(self.handle, buf, len(buf))
        check(n if n < 0 else 0)
        return np.ctypeslib.as_array(buf)[:n].reshape(-1, len(self.PHASE_STAMPS)).copy()

    def ipc_handle(self) -> bytes:
        """this rank's 64-byte handle of the layer's exchange buffer (expert
        parallelism; the layer must own only some experts)"""
        buf = (C.c_char * 64)()
        check(lib().moe_layer_ipc_handle(self.handle, buf))
        return bytes(buf)

    def set_peers(self, rank: int, handles) -> None:
        """connect the ranks: `handles` are every rank's ipc_handle(), in rank order"""
        blob = b"".join(handles)
        buf = (C.c_char * len(blob)).from_buffer_copy(blob)
        check(lib().moe_layer_set_peers(self.handle, rank, len(handles), buf))

    def status(self) -> int:
        """moe_layer_status: waits for the device and returns (and clears) the
        layer's error status as a code (0 = ok); does not raise"""
        return lib().moe_layer_status(self.handle)

    def set_wait_ms(self, ms: int) -> None:
        check(lib().moe_layer_set_wait_ms(self.handle, ms))

    def ep_reset(self) -> None:
        check(lib().moe_layer_ep_reset(self.handle))

    def routing(self, T: int, world: int = 1):
        """routing of the last forward; `world` > 1 after a token-sharded
        forward, whose dispatch covers every rank's T tokens"""
        K, NE = self.top_k, self.n_experts
        ids = np.empty((T, K), np.int32)
        w = np.empty((T, K), np.float32)
        counts = np.empty(NE, np.int32)
        offsets = np.empty(NE + 1, np.int32)
        perm = np.empty(world * T * K, np.int32)
        check(lib().moe_layer_routing(self.handle, ids.ctypes.data, w.ctypes.data,
                                      counts.ctypes.data, offsets.ctypes.data, perm.ctypes.data))
        return ids, w, counts, offsets, perm

    def close(self):
        if getattr(self, "handle", None):
            lib().moe_layer_destroy(self.handle)
            self.handle = None
        for b in self.bufs:
            b.free()
        self.bufs = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------ drop-ins
def ffn_forward(x, router_w, gate, up, down, qtype, top_k, flags=0):
    """moe_ffn_forward through tensor_t views of host arrays (OLMoE 3-D layout)."""
    x = np.ascontiguousarray(x, np.float32)
    T, d = x.shape
    NE, F = gate.shape[0], gate.shape[1]
    out = np.zeros((T, d), np.float32)
    ti, to = tensor(x), tensor(out)
    tr = tensor(np.ascontiguousarray(router_w, np.float32))
    qg, qd = qtype & 0xFF, (qtype >> 8) or (qtype & 0xFF)
    tg = tensor(gate, qg, (NE, F, d))
    tu = tensor(up, qg, (NE, F, d))
    td = tensor(down, qd, (NE, d, F))
    check(lib().moe_ffn_forward(C.byref(ti), C.byref(to), C.byref(tr), C.byref(tg),
                                C.byref(tu), C.byref(td), top_k, flags))
    return out


def ffn_forward_split(x, router_w, gates, ups, downs, qtype, top_k, flags=0):
    """moe_ffn_forward_split: Mixtral per-expert 2-D tensors."""
    x = np.ascontiguousarray(x, np.float32)
    T, d = x.shape
    NE = len(gates)
    F = gates[0].shape[0]
    out = np.zeros((T, d), np.float32)
    ti, to = tensor(x), tensor(out)
    tr = tensor(np.ascontiguousarray(router_w, np.float32))
    tg = [tensor(np.ascontiguousarray(g), qtype, (F, d)) for g in gates]
    tu = [tensor(np.ascontiguousarray(u), qtype, (F, d)) for u in ups]
    tdn = [tensor(np.ascontiguousarray(dn), qtype, (d, F)) for dn in downs]
    arr = lambda ts: (C.POINTER(MoeTensor) * NE)(*[C.pointer(t) for t in ts])  # noqa: E731
    check(lib().moe_ffn_forward_split(C.byref(ti), C.byref(to), C.byref(tr), arr(tg), arr(tu),
                                      arr(tdn), NE, top_k, flags))
    return out


def mma_transposed(lhs: np.ndarray, rhs: np.ndarray, qtype: int, n: int, k: int, add=None):
    """moe_tensor_mma_transposed_2x2_status: lhs [m,k] fp32 . rhs[n,k]^T (+ add)."""
    lhs = np.ascontiguousarray(lhs, np.float32)
    m = lhs.shape[0]
    ret = np.zeros((m, n), np.float32)
    tr = tensor(ret)
    tl = tensor(lhs)
    trh = tensor(rhs, qtype, (n, k)) if qtype != F32 else tensor(np.ascontiguousarray(rhs, np.float32))
    ta = tensor(np.ascontiguousarray(add, np.float32)) if add is not None else None
    check(lib().moe_tensor_mma_transposed_2x2_status(C.byref(tr), C.byref(tl), C.byref(trh),
                                                     C.byref(ta) if ta is not None else None))
    return ret


def fused_ffn_silu(x: np.ndarray, gate, up, down, qtype, d_ff):
    """moe_fused_ffn_silu on one token; returns (out [d], hidden [d_ff], rc)."""
    x = np.ascontiguousarray(x, np.float32).reshape(1, -1)
    d = x.shape[1]
    out = np.zeros((1, d), np.float32)
    g = np.zeros((1, d_ff), np.float32)
    u = np.zeros((1, d_ff), np.float32)
    ts = [tensor(x), tensor(out), tensor(g), tensor(gate, qtype, (d_ff, d)), tensor(u),
          tensor(up, qtype, (d_ff, d)), tensor(down, qtype, (d, d_ff))]
    rc = lib().moe_fused_ffn_silu(*[C.byref(t) for t in ts])
    return out[0], g[0], rc


def gemv_device(w_ptr, qtype, rows, cols, x_ptr, m, y_ptr, stream=None):
    check(lib().moe_gemv_device(w_ptr, qtype, rows, cols, x_ptr, m, y_ptr, stream))


def gemv(w: np.ndarray, qtype: int, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
    bw = DeviceBuffer.from_numpy(w)
    bx = DeviceBuffer.from_numpy(x)
    by = DeviceBuffer(x.shape[0] * rows * 4)
    gemv_device(bw.ptr, qtype, rows, cols, bx.ptr, x.shape[0], by.ptr)
    check(lib().moe_sync())
    return by.to_numpy(np.float32, (x.shape[0], rows))


# ------------------------------------------------------------------ whole model
class Model:
    """A device-resident OLMoE / llama-Mixtral model (moe_model_*): the
    transformer of models/olmoe/olmoe.c or models/llama/llama.c around this
    library's MoE layers.  Built from the tensor views of a GGUF file (the
    reference's loader makes the same views) or of numpy arrays."""

    def __init__(self, desc: ModelDesc, keep):
        self._keep = keep
        h = C.c_void_p()
        check(lib().moe_model_create(C.byref(h), C.byref(desc)))
        self.h = h
        self.d_model = desc.d_model
        self.vocab = desc.vocab
        self.context = desc.context

    @classmethod
    def from_gguf(cls, reader) -> "Model":
        """every tensor the model code asks gguf.c for (olmoe.c:163-183,
        llama.c:135-175), by name, from a llm.c_b200.gguf.GGUFReader"""
        def get(name):
            arr, dt, dims = reader.tensor(name)
            return tensor(arr, dt, dims)
        return cls.build(reader.kv, get)

    @classmethod
    def build(cls, kv: dict, get) -> "Model":
        """from GGUF metadata `kv` and get(name) -> MoeTensor (host or
        device payload)"""
        arch = kv["general.architecture"]
        a = arch
        L = kv[f"{a}.block_count"]
        d = kv[f"{a}.embedding_length"]
        H = kv[f"{a}.attention.head_count"]
        kvh = kv.get(f"{a}.attention.head_count_kv", H)
        ne = kv.get(f"{a}.expert_count", 0)
        keep = []

        def t(name):
            mt = get(name)
            keep.append(mt)
            return C.pointer(mt)

        def arr(names):
            ptrs = (C.POINTER(MoeTensor) * len(names))(*[t(n) for n in names])
            keep.append(ptrs)
            return C.cast(ptrs, _TPP)

        blk = lambda fmt: [fmt.format(i) for i in range(L)]  # noqa: E731
        desc = ModelDesc()
        desc.arch = ARCH_OLMOE if arch == "olmoe" else ARCH_LLAMA
        desc.n_layers, desc.d_model, desc.n_heads, desc.n_kv_heads = L, d, H, kvh
        desc.head_len = d // H
        desc.vocab = kv.get("vocab") or len(kv["tokenizer.ggml.tokens"])
        desc.context = kv[f"{a}.context_length"]
        if arch != "olmoe":
            desc.context = min(desc.context, 8192)   # llama.c:92-94
        desc.n_experts = ne
        desc.top_k = kv.get(f"{a}.expert_used_count", 0)
        desc.d_ff = kv[f"{a}.feed_forward_length"]
        desc.rope_theta = kv[f"{a}.rope.freq_base"]
        desc.token_embd = t("token_embd.weight")
        desc.output = t("output.weight")
        desc.output_norm = t("output_norm.weight")
        desc.attn_norm = arr(blk("blk.{}.attn_norm.weight"))
        desc.attn_q = arr(blk("blk.{}.attn_q.weight"))
        desc.attn_k = arr(blk("blk.{}.attn_k.weight"))
        desc.attn_v = arr(blk("blk.{}.attn_v.weight"))
        desc.attn_output = arr(blk("blk.{}.attn_output.weight"))
        desc.ffn_norm = arr(blk("blk.{}.ffn_norm.weight"))
        if arch == "olmoe":
            desc.attn_q_norm = arr(blk("blk.{}.attn_q_norm.weight"))
            desc.attn_k_norm = arr(blk("blk.{}.attn_k_norm.weight"))
            for f in ("gate", "up", "down"):
                setattr(desc, f"ffn_{f}", arr(blk("blk.{}.ffn_" + f + "_exps.weight")))
        elif ne:
            for f in ("gate", "up", "down"):
                setattr(desc, f"ffn_{f}", arr([f"blk.{i}.ffn_{f}.{e}.weight"
                                               for i in range(L) for e in range(ne)]))
        else:
            for f in ("gate", "up", "down"):
                setattr(desc, f"ffn_{f}", arr(blk("blk.{}.ffn_" + f + ".weight")))
        if ne:
            desc.ffn_gate_inp = arr(blk("blk.{}.ffn_gate_inp.weight"))
        return cls(desc, keep)

    def prefill(self, tokens, positions=None, rows=True):
        tok = np.ascontiguousarray(tokens, np.int32)
        pos = (np.arange(tok.size, dtype=np.int32) if positions is None
               else np.ascontiguousarray(positions, np.int32))
        out = np.empty((tok.size, self.d_model), np.float32) if rows else None
        check(lib().moe_model_prefill(self.h, tok.ctypes.data, pos.ctypes.data, tok.size,
                                      None if out is None else out.ctypes.data))
        return out

    def decode(self, tok: int, pos: int, row=True):
        out = np.empty(self.d_model, np.float32) if row else None
        check(lib().moe_model_decode(self.h, int(tok), int(pos),
                                     None if out is None else out.ctypes.data))
        return out

    def logits(self, row: int = 0) -> np.ndarray:
        out = np.empty(self.vocab, np.float32)
        check(lib().moe_model_logits(self.h, row, out.ctypes.data))
        return out

    def generate(self, prompt, n: int, eos: int = -1) -> np.ndarray:
        tok = np.ascontiguousarray(prompt, np.int32)
        out = np.empty(n + 1, np.int32)
        made = lib().moe_model_generate(self.h, tok.ctypes.data, tok.size, n, eos,
                                        out.ctypes.data)
        if made < 0:
            check(made)
        return out[:made]

    def reset(self):
        check(lib().moe_model_reset(self.h))

    def timing(self):
        """(prefill ms, decode ms) of the last generate, CUDA events"""
        a, b = C.c_float(), C.c_float()
        check(lib().moe_model_timing(self.h, C.byref(a), C.byref(b)))
        return a.value, b.value

    def status(self):
        return lib().moe_model_status(self.h)

    def mode(self) -> dict:
        v = lib().moe_model_mode(self.h)
        if v < 0:
            check(v)
        return {"graph": bool(v & 1), "fused": bool(v & 2), "pdl": bool(v & 4)}

    def info(self):
        cs, pos, nb = C.c_int64(), C.c_int64(), C.c_size_t()
        check(lib().moe_model_info(self.h, C.byref(cs), C.byref(pos), C.byref(nb)))
        return cs.value, pos.value, nb.value

    def close(self):
        if getattr(self, "h", None):
            lib().moe_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
