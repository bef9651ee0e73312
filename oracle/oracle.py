"""ctypes binding of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Loads oracle/liboracle.so (the C restatement of the reference's MoE FFN
path, see oracle.h) and, through a child process, the reference's own
sources compiled into oracle/_ref/.  Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline legs may import this module; the product
(llm.c_b200) never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")

F32, Q8_0, Q4_0 = 0, 1, 2
TOPK_REF, TOPK_EXACT = 0, 1

_lib = None


def build():
    """Compile liboracle.so (and oracle/_ref when the reference exists)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P = C.c_void_p
        sz = C.c_size_t
        L.orc_mix64.restype = C.c_uint64
        L.orc_mix64.argtypes = [C.c_uint64]
        L.orc_stream_seed.restype = C.c_uint64
        L.orc_stream_seed.argtypes = [C.c_uint64, C.c_uint64]
        L.orc_gauss.argtypes = [C.c_uint64, C.c_uint64, sz, C.c_float, P]
        L.orc_zipf_bias.argtypes = [C.c_uint64, sz, C.c_double, P]
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_f32_to_f16_rne.restype = C.c_uint16
        L.orc_f32_to_f16_rne.argtypes = [C.c_float]
        L.orc_f32_to_f16_trunc.restype = C.c_uint16
        L.orc_f32_to_f16_trunc.argtypes = [C.c_float]
        L.orc_quantize_row_q8_0.argtypes = [P, P, sz]
        L.orc_quantize_row_q4_0.argtypes = [P, P, sz]
        L.orc_quantize_matrix.argtypes = [C.c_int, P, sz, sz, P]
        L.orc_row_bytes.restype = sz
        L.orc_row_bytes.argtypes = [C.c_int, sz]
        L.orc_dequant_row.argtypes = [P, C.c_int, sz, P, sz]
        L.orc_dot_f32_quant.restype = C.c_float
        L.orc_dot_f32_quant.argtypes = [P, P, C.c_int, sz, sz, C.c_int]
        L.orc_dot_f32_f32.restype = C.c_float
        L.orc_dot_f32_f32.argtypes = [P, P, sz, C.c_int]
        L.orc_router_logits.argtypes = [P, sz, sz, P, sz, C.c_int, P]
        L.orc_softmax_1d.argtypes = [P, sz, C.c_int]
        L.orc_top_k.argtypes = [P, sz, P, P, sz, C.c_int]
        L.orc_dispatch.argtypes = [P, sz, sz, sz, P, P, P]
        L.orc_fused_ffn_silu.argtypes = [P, sz, sz, C.c_int, P, P, P, C.c_int, P, P]
        L.orc_gemm_q.argtypes = [P, sz, sz, P, C.c_int, sz, C.c_int, P]
        L.orc_moe_ffn.argtypes = [C.POINTER(MoeLayer), P, sz, P, P, P, P]
        L.orc_moe_slot_terms.argtypes = [C.POINTER(MoeLayer), P, sz, sz, sz, P, P, P]
        _lib = L
    return _lib


class MoeLayer(C.Structure):
    _fields_ = [
        ("d_model", C.c_size_t), ("d_ff", C.c_size_t), ("n_experts", C.c_size_t),
        ("top_k", C.c_size_t), ("qtype", C.c_int), ("renorm", C.c_int),
        ("topk_mode", C.c_int), ("lanes", C.c_int),
        ("router_w", C.c_void_p), ("router_bias", C.c_void_p),
        ("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p),
        ("gate_stride", C.c_size_t), ("up_stride", C.c_size_t), ("down_stride", C.c_size_t),
    ]


def _p(a):
    return None if a is None else a.ctypes.data


# ---------------------------------------------------------------- generator
def stream_seed(seed: int, tag: int) -> int:
    return lib().orc_stream_seed(seed, tag)


def gauss(seed: int, tag: int, n: int, sd: float, offset: int = 0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_gauss(stream_seed(seed, tag), offset, n, sd, _p(out))
    return out


def zipf_bias(seed: int, n: int, s: float = 1.1) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_zipf_bias(seed, n, s, _p(out))
    return out


# ---------------------------------------------------------------- quant
def row_bytes(qtype: int, cols: int) -> int:
    return {Q8_0: cols // 32 * 34, Q4_0: cols // 32 * 18, F32: cols * 4}[qtype]


def quantize(qtype: int, x: np.ndarray) -> np.ndarray:
    """x [..., cols] fp32 -> uint8 [..., row_bytes] in GGUF block layout."""
    x = np.ascontiguousarray(x, np.float32)
    cols = x.shape[-1]
    rows = x.size // cols
    out = np.empty(x.shape[:-1] + (row_bytes(qtype, cols),), np.uint8)
    lib().orc_quantize_matrix(qtype, _p(x), rows, cols, _p(out))
    return out


def dequant(qtype: int, q: np.ndarray, cols: int) -> np.ndarray:
    q = np.ascontiguousarray(q)
    rows = q.size // row_bytes(qtype, cols)
    out = np.empty((rows, cols), np.float32)
    for r in range(rows):
        lib().orc_dequant_row(_p(q), qtype, r, out[r].ctypes.data, cols)
    return out.reshape(q.shape[:-1] + (cols,))


def dot_f32_quant(x, q, qtype, row, n, lanes=16) -> float:
    x = np.ascontiguousarray(x, np.float32)
    return lib().orc_dot_f32_quant(_p(x), _p(np.ascontiguousarray(q)), qtype, row, n, lanes)


def gemm_q(a: np.ndarray, b: np.ndarray, qtype: int, n: int, lanes=16) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    m, k = a.shape
    c = np.empty((m, n), np.float32)
    lib().orc_gemm_q(_p(a), m, k, _p(np.ascontiguousarray(b)), qtype, n, lanes, _p(c))
    return c


# ---------------------------------------------------------------- router
def router_logits(x, wr, lanes=16) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    wr = np.ascontiguousarray(wr, np.float32)
    T, d = x.shape
    NE = wr.shape[0]
    out = np.empty((T, NE), np.float32)
    lib().orc_router_logits(_p(x), T, d, _p(wr), NE, lanes, _p(out))
    return out


def softmax(v, lanes=16) -> np.ndarray:
    v = np.array(v, np.float32, copy=True)
    for row in v.reshape(-1, v.shape[-1]):
        lib().orc_softmax_1d(row.ctypes.data, row.size, lanes)
    return v


def top_k(v, k, mode=TOPK_REF):
    v = np.ascontiguousarray(v, np.float32)
    ids = np.empty(k, np.int32)
    vals = np.empty(k, np.float32)
    lib().orc_top_k(_p(v), v.size, _p(ids), _p(vals), k, mode)
    return ids, vals


def dispatch(ids: np.ndarray, n_experts: int):
    ids = np.ascontiguousarray(ids, np.int32)
    T, k = ids.shape
    counts = np.empty(n_experts, np.int32)
    offsets = np.empty(n_experts + 1, np.int32)
    perm = np.empty(T * k, np.int32)
    lib().orc_dispatch(_p(ids), T, k, n_experts, _p(counts), _p(offsets), _p(perm))
    return counts, offsets, perm


# ---------------------------------------------------------------- layer
def moe_ffn(layer: dict, x: np.ndarray, lanes=16, topk_mode=TOPK_REF):
    """layer: dict with router_w [NE,d] f32, gate/up [NE,F,rb] u8, down [NE,d,rb] u8,
    qtype, top_k, renorm, optional router_bias.  Returns out, ids, weights, probs."""
    x = np.ascontiguousarray(x, np.float32)
    T, d = x.shape
    gate, up, down = (np.ascontiguousarray(layer[k]) for k in ("gate", "up", "down"))
    NE = gate.shape[0]
    F = layer["d_ff"]
    K = layer["top_k"]
    rb = layer.get("router_bias")
    keep = [x, gate, up, down, layer["router_w"], rb]
    L = MoeLayer(d, F, NE, K, layer["qtype"], int(layer.get("renorm", 0)), topk_mode, lanes,
                 _p(layer["router_w"]), _p(rb), _p(gate), _p(up), _p(down),
                 gate[0].nbytes, up[0].nbytes, down[0].nbytes)
    out = np.empty((T, d), np.float32)
    ids = np.empty((T, K), np.int32)
    w = np.empty((T, K), np.float32)
    probs = np.empty((T, NE), np.float32)
    lib().orc_moe_ffn(C.byref(L), _p(x), T, _p(out), _p(ids), _p(w), _p(probs))
    del keep
    return out, ids, w, probs


def moe_slot_terms(layer: dict, x: np.ndarray, first: int, nlocal: int, lanes=16,
                   topk_mode=TOPK_REF):
    """z [T*K, d]: the combine terms y / (1 / w) of the (token, slot) pairs whose
    expert is in [first, first + nlocal), zero rows elsewhere; summing a token's
    rows in slot order from 0 gives moe_ffn's output bit for bit."""
    x = np.ascontiguousarray(x, np.float32)
    T, d = x.shape
    gate, up, down = (np.ascontiguousarray(layer[k]) for k in ("gate", "up", "down"))
    NE = gate.shape[0]
    F = layer["d_ff"]
    K = layer["top_k"]
    rb = layer.get("router_bias")
    keep = [x, gate, up, down, layer["router_w"], rb]
    L = MoeLayer(d, F, NE, K, layer["qtype"], int(layer.get("renorm", 0)), topk_mode, lanes,
                 _p(layer["router_w"]), _p(rb), _p(gate), _p(up), _p(down),
                 gate[0].nbytes, up[0].nbytes, down[0].nbytes)
    z = np.zeros((T * K, d), np.float32)
    ids = np.empty((T, K), np.int32)
    w = np.empty((T, K), np.float32)
    lib().orc_moe_slot_terms(C.byref(L), _p(x), T, first, nlocal, _p(z), _p(ids), _p(w))
    del keep
    return z, ids, w


def combine_slot_terms(z: np.ndarray, T: int, K: int) -> np.ndarray:
    """out[t] = sum over slots s (in order, from 0) of z[t*K + s]"""
    z = z.reshape(T, K, -1)
    out = np.zeros((T, z.shape[2]), np.float32)
    for s in range(K):
        out = out + z[:, s]
    return out


def make_layer(seed: int, d: int, F: int, NE: int, K: int, qtype: int = Q8_0,
               renorm: bool = False, zipf: bool = False, sd: float = 0.02) -> dict:
    """Seeded synthetic MoE layer (generator tags: router 1, gate 2, up 3, down 4)."""
    wr = gauss(seed, 1, NE * d, sd).reshape(NE, d)
    gate = quantize(qtype, gauss(seed, 2, NE * F * d, sd).reshape(NE, F, d))
    up = quantize(qtype, gauss(seed, 3, NE * F * d, sd).reshape(NE, F, d))
    down = quantize(qtype, gauss(seed, 4, NE * d * F, sd).reshape(NE, d, F))
    layer = dict(router_w=wr, gate=gate, up=up, down=down, qtype=qtype, d_model=d,
                 d_ff=F, n_experts=NE, top_k=K, renorm=int(renorm))
    if zipf:
        layer["router_bias"] = zipf_bias(seed, NE, 1.1)
    return layer


def make_tokens(seed: int, T: int, d: int) -> np.ndarray:
    return gauss(seed, 5, T * d, 1.0).reshape(T, d)


# ---------------------------------------------------------------- reference (child process)
def ref_available(variant: str = "avx512") -> bool:
    return os.path.exists(os.path.join(REF_DIR, f"libref_{variant}.so"))


def ref_call(op: str, variant: str = "avx512", timeout: float = 600, **arrays) -> dict:
    """Run one reference op in a child process (the reference's thread pool
    spins on every core once its library is loaded)."""
    with tempfile.TemporaryDirectory() as td:
        fin = os.path.join(td, "in.npz")
        fout = os.path.join(td, "out.npz")
        np.savez(fin, **{k: np.asarray(v) for k, v in arrays.items()})
        subprocess.run([sys.executable, os.path.join(HERE, "ref_runner.py"), op, variant, fin, fout],
                       check=True, timeout=timeout)
        with np.load(fout) as z:
            return {k: z[k] for k in z.files}
