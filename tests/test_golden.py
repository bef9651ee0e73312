"""Golden fixtures written by the reference itself (tests/golden/make_golden.py
ran the reference's sources compiled into oracle/_ref on seeded inputs).

CPU: the oracle restatement reproduces them bit for bit (so the oracle is
pinned even where the reference sources are absent).  GPU: the library matches
them within the north-star tolerance (ids bit-exact)."""
import hashlib
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
LAYERS = ["olmoe_small", "mixtral_small", "config0_t4"]


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


_cache = {}


def load_case(orc, name):
    if name in _cache:
        return _cache[name]
    z = dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))
    c = {k: int(z[k]) for k in ("seed", "d", "F", "NE", "K", "qt", "renorm", "T")}
    c["zipf"] = bool(z["zipf"])
    L = orc.make_layer(c["seed"], c["d"], c["F"], c["NE"], c["K"], c["qt"], renorm=c["renorm"],
                       zipf=c["zipf"])
    assert digest(L["router_w"], L["gate"], L["up"], L["down"]) == str(z["weights_sha256"]), \
        "input generator drifted"
    x = orc.make_tokens(c["seed"], 32 if name == "config0_t4" else c["T"], c["d"])[:c["T"]]
    _cache[name] = (c, L, x, z)
    return _cache[name]


@pytest.mark.parametrize("name", LAYERS)
def test_oracle_reproduces_reference_golden(orc, name):
    c, L, x, z = load_case(orc, name)
    out, ids, w, _ = orc.moe_ffn(L, x)
    np.testing.assert_array_equal(ids, z["ids"])
    np.testing.assert_array_equal(w, z["w"])
    np.testing.assert_array_equal(out, z["out"])


def test_oracle_reproduces_config1_gemv_golden(orc):
    z = np.load(os.path.join(GOLDEN, "config1_gemv.npz"))
    w = orc.quantize(orc.Q4_0, orc.gauss(1, 7, 14336 * 4096, 0.02).reshape(14336, 4096))
    x = orc.gauss(1, 8, 4096, 1.0)
    assert digest(w) == str(z["weights_sha256"]) and digest(x) == str(z["x_sha256"])
    np.testing.assert_array_equal(orc.gemm_q(x[None], w, orc.Q4_0, 14336)[0], z["y"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", LAYERS)
def test_gpu_matches_reference_golden(moe, orc, name):
    from test_gpu_moe import assert_output_close
    c, L, x, z = load_case(orc, name)
    lay = moe.Layer(c["d"], c["F"], c["NE"], c["K"], c["qt"], L["router_w"], L["gate"], L["up"],
                    L["down"], router_bias=L.get("router_bias"),
                    flags=moe.RENORM if c["renorm"] else 0)
    got = lay.forward(x)
    ids, w, *_ = lay.routing(c["T"])
    np.testing.assert_array_equal(ids, z["ids"])
    np.testing.assert_allclose(w, z["w"], rtol=2.5e-7, atol=0)
    assert_output_close(got, z["out"])
    lay.close()
