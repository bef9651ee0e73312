"""The whole model on the device (moe_model_*: embedding, RMSNorm, QK-norm,
RoPE, KV cache, causal attention, MoE FFN, lm_head, greedy pick) against the
reference's own OLMoE and llama/Mixtral forward (models/olmoe/olmoe.c,
models/llama/llama.c compiled into oracle/_ref/libref_model.so) on the same
synthetic GGUF file.

Tolerance: the final-normed rows and the logits within max-abs 2e-3 and
rel-L2 1e-3 of the reference (the layer bar, applied to the whole stack);
greedy picks identical up to the first step where the reference's two best
logits are closer than 1e-3 (a near-tie either side may break)."""
import numpy as np
import pytest

from test_gguf import gguf_module

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3


def close(got, want, what):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want).max()
    rel = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    assert err <= ATOL and rel <= RTOL, f"{what}: max-abs {err:.3g} rel-L2 {rel:.3g}"


def ref_model(orc, path, tokens, n_decode, d, vocab, forced=None):
    if not orc.ref_available("model"):
        pytest.skip("oracle/_ref/libref_model.so not built")
    kw = dict(path=path, tokens=np.asarray(tokens, np.int32), n_decode=n_decode, d_model=d,
              vocab=vocab)
    if forced is not None:
        kw["forced"] = np.asarray(forced, np.int32)
    return orc.ref_call("model", "model", timeout=1800, **kw)


def same_greedy(got, ref_tokens, ref_logits):
    """picks equal until the reference's first near-tie"""
    for i, t in enumerate(ref_tokens):
        top2 = np.sort(ref_logits[i])[-2:]
        if top2[1] - top2[0] < 1e-3:
            return
        assert got[i] == t, f"pick {i}: {got[i]} != {t}"


def small_olmoe(tmp_path, context=64, layers=2, qtype=None):
    gg = gguf_module()
    path = str(tmp_path / "olmoe.gguf")
    kw = {} if qtype is None else dict(qtype=qtype)
    gg.write_olmoe(path, layers, 512, 4, 16, 4, 256, 1000, seed=21, context=context,
                   norm_sd=0.1, **kw)
    return gg, path


def test_olmoe_prefill_decode_match_reference(moe, orc, tmp_path):
    gg, path = small_olmoe(tmp_path)
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, 1000, 20)
    ref = ref_model(orc, path, prompt, 6, 512, 1000)
    model = moe.Model.from_gguf(gg.GGUFReader(path))
    rows = model.prefill(prompt)
    close(rows, ref["rows"], "prefill rows")
    close(model.logits(19), ref["logits"][0], "prefill logits")
    # teacher-forced decode with the reference's picks
    for i, t in enumerate(ref["tokens"]):
        row = model.decode(int(t), 20 + i)
        close(row, ref["drows"][i], f"decode row {i}")
        close(model.logits(0), ref["logits"][i + 1], f"decode logits {i}")
    assert model.status() == 0
    cache, _, nbytes = model.info()
    assert cache == 26 and nbytes > 0


def test_olmoe_generate_greedy(moe, orc, tmp_path):
    gg, path = small_olmoe(tmp_path)
    prompt = np.random.default_rng(6).integers(0, 1000, 12)
    ref = ref_model(orc, path, prompt, 10, 512, 1000)
    model = moe.Model.from_gguf(gg.GGUFReader(path))
    picks = model.generate(prompt, 10)
    assert picks.size == 11
    # ref["tokens"][i] is the pick fed to decode step i; the last pick of
    # the reference run is the argmax of its final logits
    want = np.concatenate([ref["tokens"], [int(np.argmax(ref["logits"][-1]))]])
    same_greedy(picks, want, ref["logits"])
    # eos stops the loop at the first pick equal to it (olmoe.c:572)
    model.reset()
    stop = int(picks[3])
    picks2 = model.generate(prompt, 10, eos=stop)
    first = int(np.argmax(picks == stop))
    assert picks2.size == first + 1 and np.array_equal(picks2, picks[:first + 1])


def test_olmoe_cache_rotation(moe, orc, tmp_path):
    """context 64: a 40-token prompt and 40 decode steps cross the context,
    the cache keeps its newest 32 rows (kvcache.c:29-55) and positions past
    the context become the cache size (olmoe.c:510-520)"""
    gg, path = small_olmoe(tmp_path, context=64)
    prompt = np.random.default_rng(7).integers(0, 1000, 40)
    ref = ref_model(orc, path, prompt, 40, 512, 1000)
    model = moe.Model.from_gguf(gg.GGUFReader(path))
    model.prefill(prompt, rows=False)
    for i, t in enumerate(ref["tokens"]):
        row = model.decode(int(t), 40 + i)
        close(row, ref["drows"][i], f"decode row {i}")
    # 40 + 24 rows fill the cache; it keeps 32, then 16 more steps: 48
    cache, _, _ = model.info()
    assert cache == 48


def test_mixtral_gqa_match_reference(moe, orc, tmp_path):
    """llama.c with experts: GQA (4 query heads on 2 KV heads), no QK-norm,
    renormalised top-2, per-expert tensors, Q4_0"""
    gg = gguf_module()
    path = str(tmp_path / "mixtral.gguf")
    gg.write_mixtral(path, 2, 512, 4, 2, 4, 2, 256, 800, seed=22, context=128, norm_sd=0.1)
    prompt = np.random.default_rng(8).integers(0, 800, 17)
    ref = ref_model(orc, path, prompt, 5, 512, 800)
    model = moe.Model.from_gguf(gg.GGUFReader(path))
    close(model.prefill(prompt), ref["rows"], "prefill rows")
    close(model.logits(16), ref["logits"][0], "prefill logits")
    for i, t in enumerate(ref["tokens"]):
        close(model.decode(int(t), 17 + i), ref["drows"][i], f"decode row {i}")
    assert model.status() == 0


def test_prefill_over_64_tokens_uses_gemm_paths(moe, orc, tmp_path):
    """a 100-token prompt takes the tcgen05 GEMM for the projections and the
    MoE layers (T > 64), and the tiled prefill attention"""
    gg, path = small_olmoe(tmp_path, context=256)
    prompt = np.random.default_rng(9).integers(0, 1000, 100)
    ref = ref_model(orc, path, prompt, 2, 512, 1000)
    model = moe.Model.from_gguf(gg.GGUFReader(path))
    close(model.prefill(prompt), ref["rows"], "prefill rows")
    for i, t in enumerate(ref["tokens"]):
        close(model.decode(int(t), 100 + i), ref["drows"][i], f"decode row {i}")


def test_model_errors(moe, tmp_path):
    gg, path = small_olmoe(tmp_path, context=32, layers=1)
    model = moe.Model.from_gguf(gg.GGUFReader(path))
    with pytest.raises(moe.MoeError) as e:
        model.prefill([1, 2, 1000])            # id outside the vocabulary
    assert e.value.code == -1
    with pytest.raises(moe.MoeError):
        model.prefill(np.arange(33) % 100)     # more rows than the context
    with pytest.raises(moe.MoeError):
        model.decode(-1, 0)
    with pytest.raises(moe.MoeError):
        model.logits(5)                        # no such row
    model.prefill([1, 2, 3], rows=False)       # still usable
    assert model.status() == 0


@pytest.mark.parametrize("arch", ["olmoe", "mixtral"])
def test_fused_decode_step_matches_reference(moe, orc, tmp_path, arch):
    """d_model 2048: the decode step takes the fused kernels (QKV GEMV with
    the residual add and RMSNorm in its prologue, one-launch QK-norm + RoPE +
    cache row + split attention with the merge by the last CTA of each head,
    programmatic dependent launches) inside the CUDA graph"""
    gg = gguf_module()
    path = str(tmp_path / f"{arch}.gguf")
    if arch == "olmoe":
        gg.write_olmoe(path, 2, 2048, 16, 8, 2, 256, 512, seed=31, context=256, norm_sd=0.1)
    else:
        gg.write_mixtral(path, 2, 2048, 16, 4, 4, 2, 512, 512, seed=32, context=256,
                         norm_sd=0.1)
    prompt = np.random.default_rng(10).integers(0, 512, 70)
    ref = ref_model(orc, path, prompt, 8, 2048, 512)
    model = moe.Model.from_gguf(gg.GGUFReader(path))
    close(model.prefill(prompt), ref["rows"], "prefill rows")
    for i, t in enumerate(ref["tokens"]):
        close(model.decode(int(t), 70 + i), ref["drows"][i], f"decode row {i}")
        close(model.logits(0), ref["logits"][i + 1], f"decode logits {i}")
    model.reset()
    picks = model.generate(prompt, 8)
    want = np.concatenate([ref["tokens"], [int(np.argmax(ref["logits"][-1]))]])
    same_greedy(picks, want, ref["logits"])
    assert model.status() == 0


@pytest.mark.parametrize("d,d_ff", [(512, 768), (2048, 1024)])
def test_dense_llama_match_reference(moe, orc, tmp_path, d, d_ff):
    """llama without experts (llama.c's dense_ffn, llama.c:365-391): the FFN
    runs as one expert that every token takes with weight 1"""
    gg = gguf_module()
    path = str(tmp_path / "dense.gguf")
    plan = gg.llama_dense_plan(2, d, d // 128, 2, d_ff, 600, context=64)
    gg.write_plan(path, plan, gg.Q8_0, seed=23, norm_sd=0.1)
    prompt = np.random.default_rng(11).integers(0, 600, 12)
    ref = ref_model(orc, path, prompt, 4, d, 600)
    model = moe.Model.from_gguf(gg.GGUFReader(path))
    close(model.prefill(prompt), ref["rows"], "prefill rows")
    for i, t in enumerate(ref["tokens"]):
        close(model.decode(int(t), 12 + i), ref["drows"][i], f"decode row {i}")
        close(model.logits(0), ref["logits"][i + 1], f"decode logits {i}")
    model.reset()
    picks = model.generate(prompt, 4)
    want = np.concatenate([ref["tokens"], [int(np.argmax(ref["logits"][-1]))]])
    same_greedy(picks, want, ref["logits"])
    assert model.status() == 0
