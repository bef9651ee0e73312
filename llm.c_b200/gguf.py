"""GGUF files for the MoE layers: a writer of synthetic random-init models in
the layout the llm.c engine loads, and a reader that builds device-resident
layers from a file's tensors.

The engine (hoathienvu8x/llm.c) maps GGUF v2/v3 files read-only and takes
its weights as views into the mapping (gguf.c:285-363 parses the header, the
metadata and the tensor infos; gguf.c:490-575 makes tensor_t views).  It
checks a tensor's element count only, and reshapes it to the dims its model
code asks for (outermost first), so the dims written here follow the ggml
convention (innermost first) and any order with the right count would load.

* OLMoE (general.architecture "olmoe", models/olmoe/olmoe.c:124-200): 3-D
  expert tensors blk.L.ffn_{gate,up,down}_exps.weight [NE, d_ff, d] and
  [NE, d, d_ff], router blk.L.ffn_gate_inp.weight [NE, d] fp32.
* Mixtral (general.architecture "llama" with llama.expert_count,
  models/llama/llama.c:82-175): per-expert 2-D tensors
  blk.L.ffn_{gate,up,down}.E.weight (llama.c:163-165).

Synthetic weights: N(0, sd) from numpy's PCG64 seeded generator (one stream
per model), quantized on the host with the reference quantizers' rounding
rules: Q8_0 as quantize_row_q8_0 (quant.c:62-78: d = amax/127 stored as
fp16 round-to-nearest-even, codes roundf(x * (1/d))), Q4_0 as the
reference's only Q4_0 quantizer, its test helper (test/quant.c:45-79: d =
amax/7 stored as fp16 by truncation, codes roundf(x * 7/amax) + 8 clamped to
0..15, element j in the low nibble of byte j and element j + 16 in its high
nibble).
"""
from __future__ import annotations

import mmap
import os
import struct

import numpy as np

GGUF_MAGIC = 0x46554747   # "GGUF"
ALIGN = 32                # gguf.c: GGUF_DEFAULT_ALIGNMENT
# metadata value types (gguf.c:19-33)
T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64 = 4, 5, 6, 7, 8, 9, 10
# tensor types (gguf.c:36-44) and this library's dtype codes
GGML_F32, GGML_Q4_0, GGML_Q8_0 = 0, 2, 8
F32, Q8_0, Q4_0 = 0, 1, 2
_GGML_OF = {F32: GGML_F32, Q8_0: GGML_Q8_0, Q4_0: GGML_Q4_0}
_DTYPE_OF = {v: k for k, v in _GGML_OF.items()}


# ---------------------------------------------------------------- quantizers
def _roundf(v: np.ndarray) -> np.ndarray:
    """C roundf: halves away from zero (numpy's rint rounds them to even)"""
    return np.sign(v) * np.floor(np.abs(v) + np.float32(0.5))


def _f16_trunc_bits(f: np.ndarray) -> np.ndarray:
    """fp32 -> fp16 bits by truncating the mantissa (test/quant.c:19-33)"""
    x = f.astype(np.float32).view(np.uint32)
    sign = ((x >> 16) & 0x8000).astype(np.uint32)
    exp = ((x >> 23) & 0xFF).astype(np.int64)
    man = x & 0x7FFFFF
    e16 = exp - 112
    out = sign | (np.clip(e16, 0, 31).astype(np.uint32) << 10) | (man >> 13)
    out = np.where(exp == 0, sign, out)
    out = np.where(exp == 0xFF, sign | 0x7C00 | np.where(man != 0, 0x200, 0), out)
    out = np.where((exp != 0xFF) & (e16 >= 0x1F), sign | 0x7C00, out)
    out = np.where((exp != 0) & (exp != 0xFF) & (e16 <= 0), sign, out)
    return out.astype(np.uint16)


def quantize(qtype: int, x: np.ndarray) -> np.ndarray:
    """x [..., cols] fp32 -> uint8 [..., cols/32 * block bytes], GGUF blocks"""
    x = np.ascontiguousarray(x, np.float32)
    cols = x.shape[-1]
    if cols % 32:
        raise ValueError("columns must be a multiple of 32")
    b = x.reshape(-1, 32)
    amax = np.abs(b).max(axis=1).astype(np.float32)
    if qtype == Q8_0:
        d = (amax / np.float32(127.0)).astype(np.float32)
        with np.errstate(divide="ignore"):
            idv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
        q = _roundf((b * idv[:, None]).astype(np.float32)).astype(np.int8)
        out = np.empty((b.shape[0], 34), np.uint8)
        out[:, :2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
        out[:, 2:] = q.view(np.uint8)
    elif qtype == Q4_0:
        scale = (amax / np.float32(7.0)).astype(np.float32)
        with np.errstate(divide="ignore"):
            inv = np.where(scale > 0, np.float32(7.0) / amax, np.float32(0.0)).astype(np.float32)
        q = (_roundf((b * inv[:, None]).astype(np.float32)) + 8).clip(0, 15).astype(np.uint8)
        out = np.empty((b.shape[0], 18), np.uint8)
        out[:, :2] = _f16_trunc_bits(scale).view(np.uint8).reshape(-1, 2)
        out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    else:
        raise ValueError(f"qtype {qtype}")
    return out.reshape(x.shape[:-1] + (-1,))


# ---------------------------------------------------------------- writer
class GGUFWriter:
    """GGUF v3: header, metadata, tensor infos, then the tensor data, each
    tensor at a 32-byte aligned offset from the start of the data section."""

    def __init__(self):
        self.kv = []        # (key, type, payload bytes)
        self.tensors = []   # (name, dims outermost first, ggml type, data bytes)

    @staticmethod
    def _str(s: str) -> bytes:
        b = s.encode()
        return struct.pack("<Q", len(b)) + b

    def add_u32(self, key, v):
        self.kv.append((key, T_U32, struct.pack("<I", int(v))))

    def add_f32(self, key, v):
        self.kv.append((key, T_F32, struct.pack("<f", float(v))))

    def add_str(self, key, v):
        self.kv.append((key, T_STR, self._str(v)))

    def add_i32_array(self, key, items):
        a = np.asarray(items, "<i4")
        self.kv.append((key, T_ARR, struct.pack("<IQ", T_I32, a.size) + a.tobytes()))

    def add_f32_array(self, key, items):
        a = np.asarray(items, "<f4")
        self.kv.append((key, T_ARR, struct.pack("<IQ", T_F32, a.size) + a.tobytes()))

    def add_str_array(self, key, items):
        payload = struct.pack("<IQ", T_STR, len(items)) + b"".join(self._str(s) for s in items)
        self.kv.append((key, T_ARR, payload))

    def add_tensor(self, name: str, data: np.ndarray, dtype: int, dims):
        """data: fp32 values (F32) or uint8 GGUF blocks; dims outermost first"""
        n = int(np.prod(dims))
        raw = np.ascontiguousarray(data).tobytes()
        want = n * 4 if dtype == F32 else n // 32 * (34 if dtype == Q8_0 else 18)
        if len(raw) != want:
            raise ValueError(f"{name}: {len(raw)} bytes for dims {dims}, want {want}")
        self.tensors.append((name, tuple(int(d) for d in dims), _GGML_OF[dtype], raw))

    def add_tensor_lazy(self, name: str, dtype: int, dims, fetch):
        """a tensor whose bytes fetch() returns when the file is written"""
        n = int(np.prod(dims))
        want = n * 4 if dtype == F32 else n // 32 * (34 if dtype == Q8_0 else 18)
        self.tensors.append((name, tuple(int(d) for d in dims), _GGML_OF[dtype], (want, fetch)))

    @staticmethod
    def _size(raw):
        return raw[0] if isinstance(raw, tuple) else len(raw)

    def write(self, path: str):
        head = struct.pack("<IIQQ", GGUF_MAGIC, 3, len(self.tensors), len(self.kv))
        for key, t, payload in self.kv:
            head += self._str(key) + struct.pack("<I", t) + payload
        offs, off = [], 0
        for name, dims, t, raw in self.tensors:
            offs.append(off)
            off = (off + self._size(raw) + ALIGN - 1) // ALIGN * ALIGN
        for (name, dims, t, raw), o in zip(self.tensors, offs):
            ggml_dims = dims[::-1]   # innermost first, as ggml writes them
            head += self._str(name) + struct.pack("<I", len(ggml_dims))
            head += b"".join(struct.pack("<Q", d) for d in ggml_dims)
            head += struct.pack("<IQ", t, o)
        pad = (-len(head)) % ALIGN
        with open(path, "wb") as f:
            f.write(head + b"\0" * pad)
            for (name, dims, t, raw), o in zip(self.tensors, offs):
                if isinstance(raw, tuple):
                    want, fetch = raw
                    raw = np.ascontiguousarray(fetch()).tobytes()
                    if len(raw) != want:
                        raise ValueError(f"{name}: {len(raw)} bytes, want {want}")
                f.write(raw)
                f.write(b"\0" * ((-len(raw)) % ALIGN))


def _vocab(n: int):
    return [f"<t{i}>" for i in range(n)]


def _norms(seed: int, norm_sd: float):
    """RMSNorm weights: ones (norm_sd 0, the usual init), else 1 + N(0,
    norm_sd) from a stream of their own (the other weights do not move)"""
    rng = np.random.default_rng(seed + 1000)
    if norm_sd == 0:
        return lambda n: np.ones(n, np.float32)
    return lambda n: (1.0 + rng.normal(0.0, norm_sd, size=n)).astype(np.float32)


def olmoe_plan(layers: int, d: int, heads: int, n_exp: int, top_k: int, d_ff: int, vocab: int,
               context: int = 4096, rope_theta: float = 10000.0):
    """(metadata setter, tensors) of an OLMoE-architecture file, in file
    order: (name, dims outermost first, kind) with kind "mat" (quantized
    N(0, sd)), "router" (F32 N(0, sd)) or "norm" (F32 RMSNorm weight); the
    names and shapes olmoe_load asks for (olmoe.c:163-183)"""
    def meta(w):
        w.add_str("general.architecture", "olmoe")
        for k, v in (("context_length", context), ("embedding_length", d),
                     ("attention.head_count", heads), ("block_count", layers),
                     ("expert_count", n_exp), ("expert_used_count", top_k),
                     ("feed_forward_length", d_ff)):
            w.add_u32("olmoe." + k, v)
        w.add_f32("olmoe.rope.freq_base", rope_theta)
        w.add_str_array("tokenizer.ggml.tokens", _vocab(vocab))
        w.add_u32("tokenizer.ggml.bos_token_id", 1)
        w.add_u32("tokenizer.ggml.eos_token_id", 2)
    ts = [("token_embd.weight", (vocab, d), "mat"), ("output.weight", (vocab, d), "mat"),
          ("output_norm.weight", (d,), "norm")]
    for i in range(layers):
        p = f"blk.{i}."
        ts.append((p + "attn_norm.weight", (d,), "norm"))
        for n in ("attn_q", "attn_k", "attn_v", "attn_output"):
            ts.append((p + n + ".weight", (d, d), "mat"))
        for n in ("attn_q_norm", "attn_k_norm", "ffn_norm"):
            ts.append((p + n + ".weight", (d,), "norm"))
        ts.append((p + "ffn_gate_inp.weight", (n_exp, d), "router"))
        ts.append((p + "ffn_gate_exps.weight", (n_exp, d_ff, d), "mat"))
        ts.append((p + "ffn_up_exps.weight", (n_exp, d_ff, d), "mat"))
        ts.append((p + "ffn_down_exps.weight", (n_exp, d, d_ff), "mat"))
    return meta, ts


def mixtral_plan(layers: int, d: int, q_heads: int, kv_heads: int, n_exp: int, top_k: int,
                 d_ff: int, vocab: int, context: int = 4096, rope_theta: float = 1e6):
    """the same for the llama architecture with experts (llama.c:92-175)"""
    hl = d // q_heads

    def meta(w):
        w.add_str("general.architecture", "llama")
        for k, v in (("context_length", context), ("embedding_length", d),
                     ("attention.head_count", q_heads), ("attention.head_count_kv", kv_heads),
                     ("block_count", layers), ("expert_count", n_exp),
                     ("expert_used_count", top_k), ("feed_forward_length", d_ff)):
            w.add_u32("llama." + k, v)
        w.add_f32("llama.rope.freq_base", rope_theta)
        # llama_load builds the vocabulary tables (llama.c:108 -> vocab.c:
        # 323-360): a SentencePiece ("llama") vocabulary with token types
        # and scores
        w.add_str("tokenizer.ggml.model", "llama")
        w.add_str_array("tokenizer.ggml.tokens", _vocab(vocab))
        w.add_i32_array("tokenizer.ggml.token_type", np.ones(vocab, np.int32))
        w.add_f32_array("tokenizer.ggml.scores", np.zeros(vocab, np.float32))
        w.add_u32("tokenizer.ggml.bos_token_id", 1)
        w.add_u32("tokenizer.ggml.eos_token_id", 2)
    ts = [("token_embd.weight", (vocab, d), "mat"), ("output.weight", (vocab, d), "mat"),
          ("output_norm.weight", (d,), "norm")]
    for i in range(layers):
        p = f"blk.{i}."
        ts.append((p + "attn_norm.weight", (d,), "norm"))
        ts.append((p + "attn_q.weight", (q_heads * hl, d), "mat"))
        ts.append((p + "attn_k.weight", (kv_heads * hl, d), "mat"))
        ts.append((p + "attn_v.weight", (kv_heads * hl, d), "mat"))
        ts.append((p + "attn_output.weight", (d, q_heads * hl), "mat"))
        ts.append((p + "ffn_norm.weight", (d,), "norm"))
        ts.append((p + "ffn_gate_inp.weight", (n_exp, d), "router"))
        for e in range(n_exp):
            ts.append((p + f"ffn_gate.{e}.weight", (d_ff, d), "mat"))
            ts.append((p + f"ffn_up.{e}.weight", (d_ff, d), "mat"))
            ts.append((p + f"ffn_down.{e}.weight", (d, d_ff), "mat"))
    return meta, ts


def llama_dense_plan(layers: int, d: int, q_heads: int, kv_heads: int, d_ff: int, vocab: int,
                     context: int = 4096, rope_theta: float = 5e5):
    """the llama architecture without experts (llama.c:86-94: one dense
    SwiGLU FFN per layer, blk.L.ffn_{gate,up,down}.weight)"""
    meta0, _ = mixtral_plan(layers, d, q_heads, kv_heads, 1, 1, d_ff, vocab, context, rope_theta)
    hl = d // q_heads

    def meta(w):
        meta0(w)
        # no experts: drop the expert keys the MoE plan wrote
        w.kv = [kv for kv in w.kv if kv[0] not in ("llama.expert_count", "llama.expert_used_count")]
    ts = [("token_embd.weight", (vocab, d), "mat"), ("output.weight", (vocab, d), "mat"),
          ("output_norm.weight", (d,), "norm")]
    for i in range(layers):
        p = f"blk.{i}."
        ts.append((p + "attn_norm.weight", (d,), "norm"))
        ts.append((p + "attn_q.weight", (q_heads * hl, d), "mat"))
        ts.append((p + "attn_k.weight", (kv_heads * hl, d), "mat"))
        ts.append((p + "attn_v.weight", (kv_heads * hl, d), "mat"))
        ts.append((p + "attn_output.weight", (d, q_heads * hl), "mat"))
        ts.append((p + "ffn_norm.weight", (d,), "norm"))
        ts.append((p + "ffn_gate.weight", (d_ff, d), "mat"))
        ts.append((p + "ffn_up.weight", (d_ff, d), "mat"))
        ts.append((p + "ffn_down.weight", (d, d_ff), "mat"))
    return meta, ts


def write_plan(path: str, plan, qtype: int, seed: int, sd: float = 0.02, norm_sd: float = 0.0):
    """a random-init file: numpy's PCG64 stream `seed` for the matrices and
    routers in file order, quantized on the host; RMSNorm weights from
    _norms"""
    meta, ts = plan
    rng = np.random.default_rng(seed)
    nrm = _norms(seed, norm_sd)
    w = GGUFWriter()
    meta(w)
    for name, dims, kind in ts:
        if kind == "norm":
            w.add_tensor(name, nrm(dims[0]), F32, dims)
        elif kind == "router":
            w.add_tensor(name, rng.normal(0.0, sd, size=dims).astype(np.float32), F32, dims)
        else:
            w.add_tensor(name, quantize(qtype, rng.normal(0.0, sd, size=dims).astype(np.float32)),
                         qtype, dims)
    w.write(path)


def write_plan_from(path: str, plan, qtype: int, fetch):
    """a file whose tensor bytes come from fetch(name) (numpy array: fp32
    values or uint8 blocks), called once per tensor while writing, so that
    a model held elsewhere (device memory) is written without a host copy
    of the whole of it"""
    meta, ts = plan
    w = GGUFWriter()
    meta(w)
    for name, dims, kind in ts:
        dt = F32 if kind in ("norm", "router") else qtype
        w.add_tensor_lazy(name, dt, dims, lambda name=name: fetch(name))
    w.write(path)


def write_olmoe(path: str, layers: int, d: int, heads: int, n_exp: int, top_k: int, d_ff: int,
                vocab: int, seed: int = 2, context: int = 4096, rope_theta: float = 10000.0,
                sd: float = 0.02, qtype: int = Q8_0, norm_sd: float = 0.0):
    """random-init OLMoE-architecture model (config 2: 16 layers, d 2048, 16
    heads, 64 experts top-8, d_ff 1024, vocab 50304, Q8_0, seed 2)"""
    write_plan(path, olmoe_plan(layers, d, heads, n_exp, top_k, d_ff, vocab, context,
                                rope_theta), qtype, seed, sd, norm_sd)


def write_mixtral(path: str, layers: int, d: int, q_heads: int, kv_heads: int, n_exp: int,
                  top_k: int, d_ff: int, vocab: int, seed: int = 3, context: int = 4096,
                  rope_theta: float = 1e6, sd: float = 0.02, qtype: int = Q4_0,
                  norm_sd: float = 0.0):
    """random-init Mixtral-architecture model ("llama" with experts; config 3:
    32 layers, d 4096, 32/8 heads, 8 experts top-2, d_ff 14336, vocab 32000,
    Q4_0, seed 3)"""
    write_plan(path, mixtral_plan(layers, d, q_heads, kv_heads, n_exp, top_k, d_ff, vocab,
                                  context, rope_theta), qtype, seed, sd, norm_sd)


# ---------------------------------------------------------------- reader
class GGUFReader:
    """Read-only mapping of a GGUF v2/v3 file (the engine's own loader,
    gguf.c:285-363, does the same); tensors come back as numpy views into the
    mapping: uint8 GGUF blocks or fp32 values."""

    def __init__(self, path: str):
        self._f = open(path, "rb")
        self.mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self.buf = memoryview(self.mm)
        self.pos = 0
        magic, version = struct.unpack_from("<II", self.buf, 0)
        if magic != GGUF_MAGIC or version not in (2, 3):
            raise ValueError(f"{path}: not a GGUF v2/v3 file")
        self.pos = 8
        n_tensors, n_kv = self._u64(), self._u64()
        self.kv = {}
        alignment = ALIGN
        for _ in range(n_kv):
            key = self._s()
            t = self._u32()
            self.kv[key] = self._value(t)
            if key == "general.alignment" and t == T_U32:
                alignment = self.kv[key]
        self.tensors = {}
        for _ in range(n_tensors):
            name = self._s()
            nd = self._u32()
            dims = [self._u64() for _ in range(nd)]
            t, off = self._u32(), self._u64()
            self.tensors[name] = (dims[::-1], t, off)   # dims outermost first
        self.data = (self.pos + alignment - 1) // alignment * alignment

    def _u32(self):
        v = struct.unpack_from("<I", self.buf, self.pos)[0]
        self.pos += 4
        return v

    def _u64(self):
        v = struct.unpack_from("<Q", self.buf, self.pos)[0]
        self.pos += 8
        return v

    def _s(self):
        n = self._u64()
        s = bytes(self.buf[self.pos:self.pos + n]).decode()
        self.pos += n
        return s

    _FMT = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q",
            11: "<q", 12: "<d"}

    def _value(self, t):
        if t == T_STR:
            return self._s()
        if t == T_ARR:
            et, n = self._u32(), self._u64()
            return [self._value(et) for _ in range(n)]
        fmt = self._FMT[t]
        v = struct.unpack_from(fmt, self.buf, self.pos)[0]
        self.pos += struct.calcsize(fmt)
        return v

    def tensor(self, name: str):
        """(numpy view, dtype code, dims outermost first)"""
        dims, t, off = self.tensors[name]
        n = int(np.prod(dims))
        dtype = _DTYPE_OF.get(t)
        if dtype is None:
            raise ValueError(f"{name}: ggml type {t} is not F32/Q8_0/Q4_0")
        start = self.data + off
        if dtype == F32:
            return np.frombuffer(self.buf, np.float32, n, start), dtype, dims
        nbytes = n // 32 * (34 if dtype == Q8_0 else 18)
        return np.frombuffer(self.buf, np.uint8, nbytes, start), dtype, dims

    def close(self):
        """unmap the file; while tensor views are still alive the mapping stays
        (it goes with the last of them)"""
        try:
            self.buf.release()
            self.mm.close()
        except BufferError:
            pass
        self._f.close()


def layer_from_gguf(moe, reader: GGUFReader, l: int, flags: int = 0, first_expert: int = 0,
                    n_local: int = 0):
    """A device-resident moe.Layer for block `l` of an OLMoE or Mixtral
    file: the router and the (local) experts' GGUF bytes uploaded as they
    are.  Mixtral layers get MOE_RENORM (llama.c:422-427)."""
    arch = reader.kv["general.architecture"]
    a = arch
    n_exp = reader.kv[f"{a}.expert_count"]
    top_k = reader.kv[f"{a}.expert_used_count"]
    d = reader.kv[f"{a}.embedding_length"]
    d_ff = reader.kv[f"{a}.feed_forward_length"]
    p = f"blk.{l}."
    router = reader.tensor(p + "ffn_gate_inp.weight")[0].reshape(n_exp, d)
    nl = n_local if n_local else n_exp - first_expert
    if arch == "olmoe":
        gate, qt, _ = reader.tensor(p + "ffn_gate_exps.weight")
        up = reader.tensor(p + "ffn_up_exps.weight")[0]
        down = reader.tensor(p + "ffn_down_exps.weight")[0]
        gate, up, down = (m.reshape(n_exp, -1) for m in (gate, up, down))
    else:
        qt = reader.tensor(p + "ffn_gate.0.weight")[1]
        gate = [reader.tensor(p + f"ffn_gate.{e}.weight")[0] for e in range(n_exp)]
        up = [reader.tensor(p + f"ffn_up.{e}.weight")[0] for e in range(n_exp)]
        down = [reader.tensor(p + f"ffn_down.{e}.weight")[0] for e in range(n_exp)]
        flags |= moe.RENORM
    keep = []

    def dev(mats):
        ptrs = []
        for e in range(n_exp):
            if first_expert <= e < first_expert + nl:
                b = moe.DeviceBuffer.from_numpy(np.ascontiguousarray(mats[e]))
                keep.append(b)
                ptrs.append(b.ptr)
            else:
                ptrs.append(0)
        return ptrs

    lay = moe.Layer(d, d_ff, n_exp, top_k, qt, np.ascontiguousarray(router), dev(gate), dev(up),
                    dev(down), flags=flags, first_expert=first_expert, n_local=n_local)
    lay.bufs.extend(keep)
    return lay


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="write a synthetic random-init GGUF model")
    ap.add_argument("path")
    ap.add_argument("--arch", choices=["olmoe", "mixtral"], default="olmoe")
    ap.add_argument("--layers", type=int)
    args = ap.parse_args(argv)
    if args.arch == "olmoe":   # config 2
        write_olmoe(args.path, args.layers or 16, 2048, 16, 64, 8, 1024, 50304, seed=2)
    else:                      # config 3
        write_mixtral(args.path, args.layers or 32, 4096, 32, 8, 8, 2, 14336, 32000, seed=3)
    print(os.path.getsize(args.path), "bytes")


if __name__ == "__main__":
    main()
