"""Writes tests/golden/*.npz: outputs of the REFERENCE (its own sources,
compiled into oracle/_ref by oracle/Makefile) on seeded synthetic inputs.

Run where the reference sources are present (oracle/_ref built):
    python tests/golden/make_golden.py
Inputs are regenerated from their seeds by the shared generator in
oracle/oracle.c; each fixture stores a digest of the generated weight bytes
so a generator change is caught.  Cases:
  olmoe_small   d 256, d_ff 128, 16 experts, top-4, Q8_0, Zipf bias, T 5
  mixtral_small d 512, d_ff 384, 8 experts, top-2, Q4_0, renorm, T 3
  config0_t4    BASELINE config 0 (OLMoE shape, seed 0), first 4 tokens
  config1_gemv  BASELINE config 1 (14336x4096 Q4_0, seed 1)
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import oracle as orc  # noqa: E402


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


CASES = {
    "olmoe_small": dict(seed=7, d=256, F=128, NE=16, K=4, qt=orc.Q8_0, renorm=0, zipf=True, T=5),
    "mixtral_small": dict(seed=3, d=512, F=384, NE=8, K=2, qt=orc.Q4_0, renorm=1, zipf=False, T=3),
    "config0_t4": dict(seed=0, d=2048, F=1024, NE=64, K=8, qt=orc.Q8_0, renorm=0, zipf=False, T=4),
}


def make_layer_case(name, c):
    L = orc.make_layer(c["seed"], c["d"], c["F"], c["NE"], c["K"], c["qt"], renorm=c["renorm"],
                       zipf=c["zipf"])
    x = orc.make_tokens(c["seed"], max(c["T"], 32) if name == "config0_t4" else c["T"], c["d"])
    x = x[:c["T"]]
    kw = dict(x=x, router_w=L["router_w"], gate=L["gate"], up=L["up"], down=L["down"],
              qtype=c["qt"], d_ff=c["F"], top_k=c["K"], renorm=c["renorm"])
    if c["zipf"]:
        kw["router_bias"] = L["router_bias"]
    r = orc.ref_call("moe", "avx512", **kw)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), out=r["out"], ids=r["ids"], w=r["w"],
                        weights_sha256=digest(L["router_w"], L["gate"], L["up"], L["down"]),
                        **{k: np.array(v) for k, v in c.items()})


def make_gemv():
    rows, cols = 14336, 4096
    w = orc.quantize(orc.Q4_0, orc.gauss(1, 7, rows * cols, 0.02).reshape(rows, cols))
    x = orc.gauss(1, 8, cols, 1.0)
    r = orc.ref_call("gemm", "avx512", a=x[None], b=w, qtype=orc.Q4_0, n=rows)
    np.savez_compressed(os.path.join(HERE, "config1_gemv.npz"), y=r["c"][0],
                        weights_sha256=digest(w), x_sha256=digest(x))


if __name__ == "__main__":
    if not orc.ref_available("avx512"):
        raise SystemExit("build oracle/_ref first: make -C oracle")
    for name, c in CASES.items():
        make_layer_case(name, c)
        print("wrote", name)
    make_gemv()
    print("wrote config1_gemv")
