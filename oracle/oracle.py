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

F32, Q8_0, Q4_0, Q4_K, Q6_K = 0, 1, 2, 3, 5
TOPK_REF, TOPK_EXACT = 0, 1
Q8K_BYTES = 292   # sizeof(block_q8_K)


def qtype2(gate_up: int, down: int) -> int:
    """a layer's weight types: gate/up in the low byte, down in the next"""
    return gate_up | (down << 8)

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
        L.orc_quantize_row_q8K.argtypes = [P, P, sz]
        L.orc_dot_q8K.restype = C.c_float
        L.orc_dot_q8K.argtypes = [P, P, C.c_int, sz, sz]
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
    return {Q8_0: cols // 32 * 34, Q4_0: cols // 32 * 18, Q4_K: cols // 256 * 144,
            Q6_K: cols // 256 * 210, F32: cols * 4}[qtype & 0xFF]


def random_kquant(qtype: int, rng: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    """valid Q4_K / Q6_K rows (quant.h:30-57) with random codes and scales,
    sized so the weights look like N(0, 0.02) ones: uint8 [rows, row_bytes].
    The reference has no K-quant quantizer; the parity tests need only
    well-formed blocks."""
    nb = rows * cols // 256
    if qtype == Q4_K:
        blk = np.empty((nb, 144), np.uint8)
        d = (1e-4 * rng.uniform(0.5, 1.5, nb)).astype(np.float16)
        dmin = (1e-3 * rng.uniform(0.5, 1.5, nb)).astype(np.float16)
        blk[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
        blk[:, 2:4] = dmin.view(np.uint8).reshape(nb, 2)
        blk[:, 4:16] = rng.integers(0, 256, (nb, 12), dtype=np.uint8)
        blk[:, 16:] = rng.integers(0, 256, (nb, 128), dtype=np.uint8)
    else:
        blk = np.empty((nb, 210), np.uint8)
        blk[:, :192] = rng.integers(0, 256, (nb, 192), dtype=np.uint8)
        blk[:, 192:208] = rng.integers(-60, 61, (nb, 16), dtype=np.int8).view(np.uint8)
        d = (5e-5 * rng.uniform(0.5, 1.5, nb)).astype(np.float16)
        blk[:, 208:210] = d.view(np.uint8).reshape(nb, 2)
    return blk.reshape(rows, -1)


def quantize_q8K(x: np.ndarray) -> np.ndarray:
    """quant.c:627-654: fp32 [n] (n % 256 == 0) -> block_q8_K bytes"""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.size // 256 * Q8K_BYTES, np.uint8)
    lib().orc_quantize_row_q8K(_p(x), _p(out), x.size)
    return out


def dot_q8K(q8: np.ndarray, q: np.ndarray, qtype: int, row: int, n: int) -> float:
    return lib().orc_dot_q8K(_p(np.ascontiguousarray(q8)), _p(np.ascontiguousarray(q)), qtype,
                             row, n)


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


def make_layer_kquant(seed: int, d: int, F: int, NE: int, K: int, gate_up: int = Q4_K,
                      down: int = Q6_K, renorm: bool = False) -> dict:
    """A MoE layer with K-quant experts (random well-formed blocks; gate/up
    and down types as in the reference's Q4_K_M files) and a seeded router"""
    rng = np.random.default_rng(seed)
    wr = gauss(seed, 1, NE * d, 0.02).reshape(NE, d)
    gate = random_kquant(gate_up, rng, NE * F, d).reshape(NE, F, -1)
    up = random_kquant(gate_up, rng, NE * F, d).reshape(NE, F, -1)
    dn = random_kquant(down, rng, NE * d, F).reshape(NE, d, -1)
    return dict(router_w=wr, gate=gate, up=up, down=dn, qtype=qtype2(gate_up, down),
                d_model=d, d_ff=F, n_experts=NE, top_k=K, renorm=int(renorm))


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
