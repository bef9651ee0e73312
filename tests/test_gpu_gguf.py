"""Layers built from a GGUF file (llm.c_b200/gguf.py: layer_from_gguf reads
the file the way the engine's loader does and uploads the router and the
experts' GGUF bytes as they are), run on the GPU, against the oracle on the
same bytes: OLMoE's 3-D expert tensors and Mixtral's per-expert tensors
(renormalised top-2)."""
import numpy as np
import pytest

from test_gguf import gguf_module
from test_gpu_moe import assert_output_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("arch,T", [("olmoe", 5), ("olmoe", 100), ("mixtral", 3)])
def test_layer_from_gguf_matches_oracle(moe, orc, tmp_path, arch, T):
    gg = gguf_module()
    path = str(tmp_path / f"{arch}.gguf")
    if arch == "olmoe":
        gg.write_olmoe(path, 2, 2048, 16, 16, 4, 1024, 64, seed=11)
    else:
        gg.write_mixtral(path, 1, 4096, 32, 8, 8, 2, 2048, 64, seed=12)
    reader = gg.GGUFReader(path)
    l = 1 if arch == "olmoe" else 0
    lay = gg.layer_from_gguf(moe, reader, l)
    a = "olmoe" if arch == "olmoe" else "llama"
    NE, K = reader.kv[f"{a}.expert_count"], reader.kv[f"{a}.expert_used_count"]
    d, F = reader.kv[f"{a}.embedding_length"], reader.kv[f"{a}.feed_forward_length"]
    p = f"blk.{l}."
    if arch == "olmoe":
        gate = reader.tensor(p + "ffn_gate_exps.weight")[0].reshape(NE, F, -1)
        up = reader.tensor(p + "ffn_up_exps.weight")[0].reshape(NE, F, -1)
        down = reader.tensor(p + "ffn_down_exps.weight")[0].reshape(NE, d, -1)
    else:
        gate = np.stack([reader.tensor(p + f"ffn_gate.{e}.weight")[0].reshape(F, -1)
                         for e in range(NE)])
        up = np.stack([reader.tensor(p + f"ffn_up.{e}.weight")[0].reshape(F, -1)
                       for e in range(NE)])
        down = np.stack([reader.tensor(p + f"ffn_down.{e}.weight")[0].reshape(d, -1)
                         for e in range(NE)])
    qt = reader.tensor(p + ("ffn_gate_exps.weight" if arch == "olmoe" else "ffn_gate.0.weight"))[1]
    L = dict(router_w=np.array(reader.tensor(p + "ffn_gate_inp.weight")[0]).reshape(NE, d),
             gate=gate, up=up, down=down, qtype=qt, d_model=d, d_ff=F, n_experts=NE, top_k=K,
             renorm=int(arch == "mixtral"))
    x = orc.make_tokens(13, T, d)
    got = lay.forward(x)
    ref = orc.moe_ffn(L, x)[0]
    assert_output_close(got, ref)
    lay.close()
    reader.close()
