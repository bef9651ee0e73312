"""Child-process driver for the reference compiled into oracle/_ref/ (TEST
INFRASTRUCTURE ONLY).

usage: ref_runner.py OP VARIANT IN.npz OUT.npz

Loading a _ref library starts the reference's spinning thread pool, so this
runs in its own process and exits when the op is done.  Ops:
  moe      ref_moe_ffn        (x, router_w, gate, up, down, qtype, d_ff, top_k, renorm[, router_bias])
  gemm     ref_gemm           (a, b, qtype, n)
  softmax  ref_softmax        (v [rows, n])
  topk     ref_top_k          (v [rows, n], k)
  q8       ref_quantize_row_q8_0 (x [rows, n])
  dot      ref_dot_f32_quant  (x, q, qtype, n, rows)
  ffn      ref_fused_ffn_silu (x, gate, up, down, qtype, d_ff)
  bench    times ref_moe_ffn: (same as moe, plus reps) -> seconds per call
  q8k      ref_quantize_row_q8K (x [n])
  dotq8k   ref_dot_q8K        (q8, q, qtype, n, rows)
  model    (variant "model": libref_model.so) the reference's own OLMoE /
           llama-Mixtral forward on a GGUF file: prefill `tokens` at
           positions 0.., logits of the last row, then `n_decode` steps fed
           with `forced` tokens (or greedy argmax, main.c:189-193) ->
           prefill rows, per-step output rows, logits, tokens, seconds
"""
import ctypes as C
import os
import sys
import time

import numpy as np


def main():
    op, variant, fin, fout = sys.argv[1:5]
    here = os.path.dirname(os.path.abspath(__file__))
    L = C.CDLL(os.path.join(here, "_ref", f"libref_{variant}.so"))
    z = dict(np.load(fin))
    P = C.c_void_p
    sz = C.c_size_t
    p = lambda a: None if a is None else a.ctypes.data  # noqa: E731
    out = {}

    def moe_args(zz):
        x = np.ascontiguousarray(zz["x"], np.float32)
        T, d = x.shape
        wr = np.ascontiguousarray(zz["router_w"], np.float32)
        NE = wr.shape[0]
        rb = zz.get("router_bias")
        rb = None if rb is None else np.ascontiguousarray(rb, np.float32)
        K = int(zz["top_k"])
        o = np.empty((T, d), np.float32)
        ids = np.empty((T, K), np.int32)
        w = np.empty((T, K), np.float32)
        L.ref_moe_ffn.argtypes = [P, sz, sz, P, sz, P, P, P, P, C.c_int, sz, sz, C.c_int, P, P, P]
        args = [p(x), T, d, p(wr), NE, p(rb), p(zz["gate"]), p(zz["up"]), p(zz["down"]),
                int(zz["qtype"]), int(zz["d_ff"]), K, int(zz["renorm"]), p(o), p(ids), p(w)]
        return args, (x, wr, rb), o, ids, w

    if op in ("moe", "bench"):
        for k in ("gate", "up", "down"):
            z[k] = np.ascontiguousarray(z[k])
        args, keep, o, ids, w = moe_args(z)
        if op == "moe":
            rc = L.ref_moe_ffn(*args)
            assert rc == 0
            out = dict(out=o, ids=ids, w=w)
        else:
            reps = int(z.get("reps", 3))
            L.ref_moe_ffn(*args)  # warm-up
            ts = []
            for _ in range(reps):
                t0 = time.perf_counter()
                L.ref_moe_ffn(*args)
                ts.append(time.perf_counter() - t0)
            out = dict(seconds=np.array(ts), out=o, ids=ids, w=w)
    elif op == "gemm":
        a = np.ascontiguousarray(z["a"], np.float32)
        b = np.ascontiguousarray(z["b"])
        m, k = a.shape
        n = int(z["n"])
        c = np.empty((m, n), np.float32)
        L.ref_gemm.argtypes = [P, sz, sz, P, C.c_int, sz, P]
        reps = int(z.get("reps", 0))
        L.ref_gemm(p(a), m, k, p(b), int(z["qtype"]), n, p(c))
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            L.ref_gemm(p(a), m, k, p(b), int(z["qtype"]), n, p(c))
            ts.append(time.perf_counter() - t0)
        out = dict(c=c, seconds=np.array(ts))
    elif op == "model":
        L.refm_load.restype = P
        L.refm_load.argtypes = [C.c_char_p]
        L.refm_prefill.argtypes = [P, P, P, sz, P]
        L.refm_decode.argtypes = [P, C.c_int, C.c_int, P]
        L.refm_logits.argtypes = [P, P, P]
        h = L.refm_load(str(z["path"]).encode())
        assert h, "refm_load failed"
        tok = np.ascontiguousarray(z["tokens"], np.int32)
        T = tok.size
        pos = np.arange(T, dtype=np.int32)
        E, V = int(z["d_model"]), int(z["vocab"])
        nd = int(z.get("n_decode", 0))
        forced = z.get("forced")
        rows = np.empty((T, E), np.float32)
        t0 = time.perf_counter()
        assert L.refm_prefill(h, p(tok), p(pos), T, p(rows)) == 0
        t_prefill = time.perf_counter() - t0
        logits = np.empty((nd + 1, V), np.float32)
        drows = np.empty((nd, E), np.float32)
        toks = np.empty(nd, np.int32)
        L.refm_logits(h, p(rows[T - 1]), p(logits[0]))
        t_decode = 0.0
        for i in range(nd):
            # greedy: the first maximum (main.c:189-193)
            nxt = int(forced[i]) if forced is not None else int(np.argmax(logits[i]))
            toks[i] = nxt
            t0 = time.perf_counter()
            L.refm_decode(h, nxt, T + i, p(drows[i]))
            L.refm_logits(h, p(drows[i]), p(logits[i + 1]))
            t_decode += time.perf_counter() - t0
        out = dict(rows=rows, logits=logits, drows=drows, tokens=toks,
                   prefill_seconds=np.array(t_prefill), decode_seconds=np.array(t_decode))
    elif op == "softmax":
        v = np.array(z["v"], np.float32, copy=True)
        L.ref_softmax.argtypes = [P, sz]
        for row in v:
            L.ref_softmax(row.ctypes.data, row.size)
        out = dict(v=v)
    elif op == "topk":
        v = np.ascontiguousarray(z["v"], np.float32)
        k = int(z["k"])
        ids = np.empty((v.shape[0], k), np.int32)
        vals = np.empty((v.shape[0], k), np.float32)
        L.ref_top_k.argtypes = [P, sz, P, P, sz]
        for r in range(v.shape[0]):
            L.ref_top_k(v[r].ctypes.data, v.shape[1], ids[r].ctypes.data, vals[r].ctypes.data, k)
        out = dict(ids=ids, vals=vals)
    elif op == "q8k":
        x = np.ascontiguousarray(z["x"], np.float32)
        q = np.empty(x.size // 256 * 292, np.uint8)
        L.ref_quantize_row_q8K.argtypes = [P, P, sz]
        L.ref_quantize_row_q8K(p(x), p(q), x.size)
        out = dict(q=q)
    elif op == "dotq8k":
        q8 = np.ascontiguousarray(z["q8"])
        q = np.ascontiguousarray(z["q"])
        n, rows = int(z["n"]), int(z["rows"])
        L.ref_dot_q8K.restype = C.c_float
        L.ref_dot_q8K.argtypes = [P, P, C.c_int, sz, sz]
        out = dict(y=np.array([L.ref_dot_q8K(p(q8), p(q), int(z["qtype"]), r, n)
                               for r in range(rows)], np.float32))
    elif op == "q8":
        x = np.ascontiguousarray(z["x"], np.float32)
        rows, n = x.shape
        q = np.empty((rows, n // 32 * 34), np.uint8)
        L.ref_quantize_row_q8_0.argtypes = [P, P, sz]
        for r in range(rows):
            L.ref_quantize_row_q8_0(x[r].ctypes.data, q[r].ctypes.data, n)
        out = dict(q=q)
    elif op == "dot":
        x = np.ascontiguousarray(z["x"], np.float32)
        q = np.ascontiguousarray(z["q"])
        n = int(z["n"])
        rows = int(z["rows"])
        L.ref_dot_f32_quant.restype = C.c_float
        L.ref_dot_f32_quant.argtypes = [P, P, C.c_int, sz, sz]
        out = dict(y=np.array([L.ref_dot_f32_quant(p(x), p(q), int(z["qtype"]), r, n)
                               for r in range(rows)], np.float32))
    elif op == "ffn":
        x = np.ascontiguousarray(z["x"], np.float32)
        d = x.size
        o = np.empty(d, np.float32)
        L.ref_fused_ffn_silu.argtypes = [P, sz, sz, C.c_int, P, P, P, P]
        ok = L.ref_fused_ffn_silu(p(x), d, int(z["d_ff"]), int(z["qtype"]),
                                  p(np.ascontiguousarray(z["gate"])), p(np.ascontiguousarray(z["up"])),
                                  p(np.ascontiguousarray(z["down"])), p(o))
        out = dict(out=o, ok=np.array(ok))
    else:
        raise SystemExit(f"unknown op {op}")
    np.savez(fout, **out)
    sys.stdout.flush()
    # skip the reference's destructor (it joins spinning workers)
    os._exit(0)


if __name__ == "__main__":
    main()
