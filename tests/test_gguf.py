"""Synthetic GGUF models (llm.c_b200/gguf.py) against the reference's own
loader.  oracle/_ref/gguf_check is the reference's gguf.c, compiled from its
sources, reading a file the writer made: it must find every tensor the
OLMoE / Mixtral loaders ask for (olmoe.c:124-200, llama.c:82-175, the
per-expert names of llama.c:163-165 included), with the dtype, element
count and bytes the writer put there.  The writer's host quantizers must
give the reference quantizers' bytes (checked against the oracle, which is
pinned to the compiled reference)."""
import importlib.util
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CHECK = os.path.join(ROOT, "oracle", "_ref", "gguf_check")


def gguf_module():
    spec = importlib.util.spec_from_file_location("moe_gguf", os.path.join(ROOT, "llm.c_b200",
                                                                            "gguf.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def fnv1a(b: bytes) -> int:
    h = 1469598103934665603
    for x in b:
        h = ((h ^ x) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


@pytest.mark.parametrize("qt", [1, 2])
def test_host_quantizers_match_the_reference(orc, qt):
    gg = gguf_module()
    x = np.random.default_rng(7).normal(0, 0.02, (96, 512)).astype(np.float32)
    x[0, :32] = 0.0
    x[1, :32] *= 200.0
    x[2, :32] = np.float32(0.5) * np.float32(0.02)   # halves at the rounding ties
    np.testing.assert_array_equal(gg.quantize(qt, x), orc.quantize(qt, x))


@pytest.mark.parametrize("arch", ["olmoe", "mixtral"])
def test_reference_loader_reads_the_synthetic_model(tmp_path, arch):
    if not os.path.exists(CHECK):
        pytest.skip("oracle/_ref/gguf_check not built (reference sources absent)")
    gg = gguf_module()
    path = str(tmp_path / f"{arch}.gguf")
    if arch == "olmoe":
        gg.write_olmoe(path, 2, 256, 4, 8, 2, 128, 64, seed=5)
        meta = "meta olmoe E=256 L=2 NE=8 K=2 EI=128 H=4 KVH=4 V=64 theta=10000"
    else:
        gg.write_mixtral(path, 2, 256, 4, 2, 4, 2, 512, 64, seed=6)
        meta = "meta llama E=256 L=2 NE=4 K=2 EI=512 H=4 KVH=2 V=64 theta=1e+06"
    r = subprocess.run([CHECK, path], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.strip().split("\n")
    assert lines[0] == meta
    reader = gg.GGUFReader(path)
    assert len(lines) - 1 == len(reader.tensors)
    for ln in lines[1:]:
        name, t, n, h = ln.split()
        view, dtype, dims = reader.tensor(name)
        assert int(t) == dtype and int(n) == int(np.prod(dims)), ln
        assert int(h, 16) == fnv1a(view.tobytes()), ln
    reader.close()


def test_reader_round_trip(tmp_path):
    gg = gguf_module()
    path = str(tmp_path / "m.gguf")
    gg.write_olmoe(path, 1, 64, 2, 4, 2, 64, 16, seed=9)
    r = gg.GGUFReader(path)
    assert r.kv["general.architecture"] == "olmoe"
    assert r.kv["olmoe.expert_count"] == 4 and len(r.kv["tokenizer.ggml.tokens"]) == 16
    v, dtype, dims = r.tensor("blk.0.ffn_down_exps.weight")
    assert dtype == 1 and dims == [4, 64, 64] and v.nbytes == 4 * 64 * 2 * 34
    w, dtype, dims = r.tensor("blk.0.ffn_gate_inp.weight")
    assert dtype == 0 and dims == [4, 64] and w.dtype == np.float32
    r.close()
