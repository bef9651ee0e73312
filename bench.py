#!/usr/bin/env python3
"""Benchmark of the B200 MoE FFN layer (BASELINE.json metric: MoE-layer
tokens/s and achieved HBM TB/s).

Default workload = BASELINE config 0: one OLMoE-1B-7B-shaped MoE FFN layer
(d_model 2048, 64 experts, top-8 without renormalisation, d_ff 1024 SwiGLU,
Q8_0 experts, fp32 router) on T = 32 tokens per GPU.  A step is one layer
forward.  Weights are synthetic (seeded N(0, 0.02) through the shared
generator, quantized to Q8_0 on the device); NL distinct layers are rotated
so that every step streams experts that are not in the 126 MB L2.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--tokens T] [--layers NL] [--prefill-tokens P] [--no-sweeps] ...

Prints one JSON line (rank 0).  Under torchrun the layer is expert-parallel
and token-sharded: rank r holds experts expert_range(r) of every layer and
its own T tokens (rows [r*T, r*T+T) of one global batch), so the work per GPU
is fixed as N grows (weak scaling); the time is the max over ranks and the
value counts every rank's tokens.  The line also carries: the replicated-token
variant at N > 1 (every rank the same tokens, strong scaling), the prefill leg
(P tokens per GPU, the tcgen05 grouped GEMM, NCCL all-to-all at N > 1), the
config-1 GEMV, the config-3 (Mixtral-shaped) and config-4 (Zipf-skewed) token
sweeps, the reference CPU baseline on identical bytes, and a parity block
(the measured layer's output against the reference or the oracle).
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

EXPERT_BYTES_Q8 = 3 * 1024 * 2048 // 32 * 34  # 6,684,672 B per OLMoE expert


def load_package():
    if "moe_b200" in sys.modules:
        return sys.modules["moe_b200"]
    spec = importlib.util.spec_from_file_location(
        "moe_b200", os.path.join(ROOT, "llm.c_b200", "__init__.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["moe_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.out = None

    def start(self):
        try:
            self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.out, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.flush()
        rows = []
        with open(self.out.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.out.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": reasons, "samples": len(rows)}




def build_layers(moe, nl, seed0, d, F, NE, K, qtype, stream, first=0, n_local=None,
                 router_bias=None, flags=0):
    """NL device-resident layers generated on the GPU (generator tags: router
    1, gate 2, up 3, down 4; layer l uses seed seed0 + l).  Expert parallelism:
    only experts [first, first + n_local) are generated and held here, with
    the same values as in the full layer."""
    import torch
    n_local = NE if n_local is None else n_local
    rb_d = moe.row_bytes(qtype, d)
    rb_f = moe.row_bytes(qtype, F)
    layers, keep = [], []
    tmp = torch.empty(n_local * F * d, dtype=torch.float32, device="cuda")
    for l in range(nl):
        seed = seed0 + l
        wr = torch.empty(NE * d, dtype=torch.float32, device="cuda")
        moe.check(moe.lib().moe_synth_gauss(wr.data_ptr(), seed, 1, 0, NE * d, 0.02, stream))
        mats = []
        for tag, rows, cols, rb in ((2, F, d, rb_d), (3, F, d, rb_d), (4, d, F, rb_f)):
            q = torch.empty(n_local * rows * rb, dtype=torch.uint8, device="cuda")
            moe.check(moe.lib().moe_synth_gauss(tmp.data_ptr(), seed, tag, first * rows * cols,
                                                n_local * rows * cols, 0.02, stream))
            moe.check(moe.lib().moe_quantize_device(tmp.data_ptr(), n_local * rows, cols, qtype,
                                                    q.data_ptr(), stream))
            mats.append(q)
        torch.cuda.synchronize()
        ptrs = [[m.data_ptr() + (e - first) * rows_b if first <= e < first + n_local else 0
                 for e in range(NE)]
                for m, rows_b in zip(mats, (F * rb_d, F * rb_d, d * rb_f))]
        lay = moe.Layer(d, F, NE, K, qtype, wr.data_ptr(), ptrs[0], ptrs[1], ptrs[2],
                        router_bias=router_bias, flags=flags, first_expert=first,
                        n_local=n_local)
        layers.append(lay)
        keep.append((wr, mats))
    del tmp
    return layers, keep


# --------------------------------------------------------------------------- ours
DECODE_MAX_T = 64   # batches above this take the prefill GEMM path


def init_rank(world, local_rank):
    import torch
    torch.cuda.set_device(local_rank)
    moe = load_package()
    moe.init(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    # a dedicated stream: the handle of torch's default stream is 0, which the
    # library reads as "use the library stream"
    torch_stream = torch.cuda.Stream()
    torch.cuda.set_stream(torch_stream)
    return torch, moe, dist, torch_stream


def gather_fn(dist, world):
    def gather(obj):
        got = [None] * world
        dist.all_gather_object(got, obj)
        return got
    return gather


def max_over_ranks(dist, v):
    if not dist:
        return v
    import torch
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def synth_tokens(moe, torch, n_tok, d, seed, tag, first_tok, stream):
    """rows [first_tok, first_tok + n_tok) of the token stream (seed, tag)"""
    x = torch.empty(n_tok * d, dtype=torch.float32, device="cuda")
    moe.check(moe.lib().moe_synth_gauss(x.data_ptr(), seed, tag, first_tok * d, n_tok * d, 1.0,
                                        stream))
    return x


def time_graph_steps(torch, dist, torch_stream, step, NL, K, profile_flag):
    """Exactly K layer forwards (step(i, flags)) from CUDA graphs: a graph of
    NL rotated forwards replayed K // NL times plus a graph of the first
    K % NL forwards; CUDA events on the launching stream, max over ranks.
    Returns (ms for the K steps, the NL-forward graph, host enqueue ms)."""
    g_full = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_full, stream=torch_stream, capture_error_mode="relaxed"):
        for l in range(NL):
            step(l, profile_flag)
    g_full.replay()
    rem = K % NL
    g_rem = None
    if rem:
        g_rem = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_rem, stream=torch_stream, capture_error_mode="relaxed"):
            for l in range(rem):
                step(l, 0)
        g_rem.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    h0 = time.perf_counter()
    ev0.record(torch_stream)
    for _ in range(K // NL):
        g_full.replay()
    if g_rem is not None:
        g_rem.replay()
    ev1.record(torch_stream)
    host_ms = (time.perf_counter() - h0) * 1e3
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = max_over_ranks(dist, ev0.elapsed_time(ev1))
    return ms, g_full, host_ms


def time_graph_long(torch, dist, torch_stream, g_full, NL, ms_per_step, min_ms=200.0):
    """the same graph replayed for at least min_ms (a steadier figure beside
    the exact-K one)"""
    reps = max(1, int(min_ms / max(ms_per_step * NL, 1e-3)) + 1)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(torch_stream)
    for _ in range(reps):
        g_full.replay()
    ev1.record(torch_stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(dist, ev0.elapsed_time(ev1))
    return {"steps": reps * NL, "ms_per_step": ms / (reps * NL), "timed_ms": ms}


def run_ours(args, rank, world, local_rank):
    torch, moe, dist, torch_stream = init_rank(world, local_rank)
    stream = torch_stream.cuda_stream
    d, F, NE, K, qtype = 2048, 1024, 64, 8, moe.Q8_0
    T, NL = args.tokens, args.layers
    first, n_local = moe.expert_range(rank, world, NE)
    layers, keep = build_layers(moe, NL, 0, d, F, NE, K, qtype, stream, first, n_local)
    if world > 1:
        gather = gather_fn(dist, world)
        for lay in layers:
            moe.connect_expert_parallel(lay, rank, gather)
        moe.init_expert_parallel_comm(rank, world, gather)
    # N > 1: token-sharded expert parallelism.  Rank r holds experts
    # expert_range(r) of every layer and its own T tokens, rows [r*T, r*T+T)
    # of one global batch (as data-parallel attention feeds an
    # expert-parallel FFN); tokens go to the experts' ranks and rows back.
    shard = moe.EP_SHARDED if world > 1 else 0
    x = synth_tokens(moe, torch, T, d, 0, 5, rank * T, stream)   # config-0 tokens: seed 0, tag 5
    out = torch.empty(T * d, dtype=torch.float32, device="cuda")

    def step(i, flags=0):
        layers[i % NL].forward_device(x.data_ptr(), out.data_ptr(), T, shard | flags, stream)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    # routing of each layer: this rank's experts that received pairs (their
    # bytes are the algorithmic bytes) and its pairs
    uniq, pairs_local = [], []
    for l in range(NL):
        step(l)
        counts = layers[l].routing(T, world)[2]
        loc = counts[first:first + n_local]
        uniq.append(int((loc > 0).sum()))
        pairs_local.append(int(loc.sum()))
    torch.cuda.synchronize()

    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)
    ms_total, g_full, host_ms = time_graph_steps(torch, dist, torch_stream, step, NL, args.steps,
                                                 moe.PROFILE)
    ms_step = ms_total / args.steps
    long_run = time_graph_long(torch, dist, torch_stream, g_full, NL, ms_step)
    clk = clocks.stop()
    stage = np.zeros(5)
    nprof = 0
    for lay in layers:
        try:
            s, c = lay.stage_ms()
            stage += np.array(s)
            nprof += c
        except moe.MoeError:
            pass
    status = [lay.status() for lay in layers]
    del g_full
    tokens_per_s = world * T * args.steps / (ms_total / 1e3)

    # ---- roofline of the dominant kernel: the fused decode-layer kernel, one
    # launch per layer forward (router, routing, gate/up + SwiGLU, down, combine)
    hbm_peak, _, peak_kind = measured_peaks()
    U = np.array([uniq[i % NL] for i in range(args.steps)], float)
    layer_bytes = float(np.mean(U)) * EXPERT_BYTES_Q8 + NE * d * 4 + 2 * T * d * 4
    stage_avg = stage / max(nprof, 1)
    kernel_ms = float(stage_avg.sum())
    achieved = layer_bytes / (kernel_ms / 1e3) / 1e9 if kernel_ms > 0 else None
    stage_names = ["router", "routing", "gate_up", "down", "combine"]
    roof = {"bound": "hbm",
            "kernel": "moe_decode_kernel<Q8_0, 16 lanes> (whole MoE layer, one launch)",
            "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
            "frac": achieved / hbm_peak if achieved else None, "traffic": None,
            "peak_source": peak_kind + " (burst copy bandwidth)",
            "algorithmic_bytes_per_launch": layer_bytes, "avg_launch_ms": kernel_ms,
            "bytes_basis": "this rank's routed experts x 6,684,672 B + router 524,288 B + "
                           "its tokens in and out",
            "launch_time_source": "%globaltimer stamps of every CTA (earliest start to "
                                  "latest end), averaged over the profiled replays",
            "step_achieved_gbs": layer_bytes / (ms_step / 1e3) / 1e9,
            "stage_ms_avg": {n: float(v) for n, v in zip(stage_names, stage_avg)}}
    if T > DECODE_MAX_T:
        roof = dict(gemm_roofline(stage_avg, float(np.mean(pairs_local)), d, F),
                    stage_ms_avg=roof["stage_ms_avg"], step_ms=ms_step)
    traffic = os.path.join(ROOT, "profiles", "traffic.json")
    if T <= DECODE_MAX_T and world == 1 and os.path.exists(traffic):
        with open(traffic) as f:
            tj = json.load(f)
        # DRAM bytes of one captured launch, scaled by the routed experts
        per_expert, fixed = tj.get("bytes_per_active_expert"), tj.get("bytes_fixed", 0.0)
        if per_expert and tj.get("kernel") == roof["kernel"]:
            roof["traffic"] = per_expert * float(np.mean(U)) + fixed
            roof["traffic_source"] = "profiles/" + tj.get("source", "traffic.json")

    # ---- parity of the measured layer: layer 0 on this rank's tokens again,
    # checked on rank 0 (N = 1: against the reference itself, in cpu_baseline)
    layers[0].forward_device(x.data_ptr(), out.data_ptr(), T, shard, stream)
    torch.cuda.synchronize()
    out0 = out.view(T, d).cpu().numpy().copy()
    ids0 = layers[0].routing(T, world)[0]
    x_host = x.view(T, d).cpu().numpy().copy()

    # ---- replicated tokens (N > 1): every rank the same T tokens and the full
    # output (strong scaling of the same kernel), for comparison
    replicated = None
    if world > 1 and not args.no_replicated:
        xr = synth_tokens(moe, torch, T, d, 0, 5, 0, stream)

        def step_rep(i, flags=0):
            layers[i % NL].forward_device(xr.data_ptr(), out.data_ptr(), T, flags, stream)

        for i in range(max(3, NL)):
            step_rep(i)
        torch.cuda.synchronize()
        ms_rep, g_rep, _ = time_graph_steps(torch, dist, torch_stream, step_rep, NL, 4 * NL,
                                            moe.PROFILE)
        del g_rep
        st_rep = np.zeros(5)
        n_rep = 0
        for lay in layers:
            s, c = lay.stage_ms()
            st_rep += np.array(s)
            n_rep += c
        replicated = {"value": T * 4 * NL / (ms_rep / 1e3), "unit": "tokens/s",
                      "ms_per_step": ms_rep / (4 * NL), "steps": 4 * NL,
                      "scaling": "strong",
                      "stage_ms_avg": {n: float(v) for n, v in
                                       zip(stage_names, st_rep / max(n_rep, 1))},
                      "how": "every rank the same T tokens; each (token, slot) row of a rank's "
                             "experts written into every rank's exchange buffer; every rank "
                             "combines the full output"}

    # ---- e2e: the reference-facing call with host buffers (H2D + D2H inside)
    if args.no_e2e:
        e2e = None
    elif world == 1:
        e2e = run_e2e(moe, args, layers, keep, T, d, F, NE, K, qtype, rank, dist)
    else:
        e2e = run_e2e_ep(moe, args, layers, x_host, T, d, stream, dist)

    prefill = None
    if args.prefill_tokens > 0:
        prefill = run_prefill(moe, torch, args, layers, rank, world, d, F, NE, K, stream,
                              torch_stream, dist)

    gemv1, dense = None, None
    if world == 1 and not args.no_gemv:
        gemv1 = run_config1_gemv(moe, stream, torch_stream)
        dense = run_dense_gemm(moe, stream, torch_stream)

    cpu, parity = None, None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu, parity = cpu_baseline(keep[0], x_host, out0, ids0, T, d, F, NE, K, qtype)
    elif rank == 0 and not args.no_parity:
        parity = oracle_parity(x_host, out0, ids0, d, F, NE, K, args.parity_tokens)

    sweeps = {}
    if not args.no_sweeps:
        # free all but layer 0 first (no rank may still write into them)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        for lay in layers[1:]:
            lay.close()
        del layers[1:], keep[1:]
        torch.cuda.empty_cache()
        sweeps["config4"] = sweep_leg(moe, torch, dist, rank, world, torch_stream, "olmoe",
                                      [int(t) for t in args.sweep4.split(",") if t])
        sweeps["config3"] = sweep_leg(moe, torch, dist, rank, world, torch_stream, "mixtral",
                                      [int(t) for t in args.sweep3.split(",") if t],
                                      cpu_tokens=0 if (world > 1 or args.no_cpu) else 2)

    models = {}
    if world == 1 and not args.no_model:
        torch.cuda.synchronize()
        for lay in layers[1:]:
            lay.close()
        del layers[1:], keep[1:]
        torch.cuda.empty_cache()
        for cfg in [c for c in args.models.split(",") if c]:
            models[cfg] = run_model_leg(moe, torch, torch_stream, cfg, runs=args.model_runs,
                                        with_ref=not args.no_cpu, clocks_dev=local_rank,
                                        n_decode=args.model_decode)
            torch.cuda.empty_cache()

    line = {
        "metric": "MoE-layer tokens/s (OLMoE config 0, T=%d%s)" % (
            T, " per GPU" if world > 1 else ""),
        "value": tokens_per_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak" if world > 1 else "strong", "vs_baseline": None,
        "dtype": "fp32 activations x Q8_0 weights",
        "data": "synthetic (seeded N(0,0.02) weights -> Q8_0, N(0,1) tokens)",
        "config": {"workload": "config0: OLMoE-1B-7B MoE FFN layer, d 2048, 64 experts top-8, "
                               "d_ff 1024 SwiGLU, Q8_0, T=%d tokens per GPU" % T,
                   "tokens_per_step": world * T, "tokens_per_gpu": T, "layers_rotated": NL,
                   "l2": f"{NL} distinct layers rotated; each step streams "
                         f"{np.mean(U) * EXPERT_BYTES_Q8 / 1e6:.0f} MB of experts per GPU "
                         f"(> 126 MB L2 over the rotation)",
                   "parallelism": (f"expert-parallel x{world}, token-sharded: {n_local} experts "
                                   f"and {T} tokens per GPU; tokens and top-k ids to every rank "
                                   "and each (token, slot) row back to its token's rank over "
                                   "NVLink inside the fused kernel")
                                  if world > 1 else "single GPU"},
        "e2e": e2e, "roofline": roof, "cpu_baseline": cpu, "parity": parity, "clocks": clk,
        # one fused decode-layer kernel per forward; above 64 tokens: router,
        # top-k + dispatch (one launch up to 256 tokens, two above), gather,
        # two GEMMs and the combine
        "gpu_launches": args.steps * (1 if T <= DECODE_MAX_T else 6 if T <= 256 else 7),
        "host_enqueue_ms": host_ms,
        "timing": "CUDA events on the launching stream around CUDA-graph replays: exactly "
                  f"{args.steps} layer forwards ({NL} rotated layers per graph, plus a graph "
                  "of the remainder), max over ranks",
        "long_timing": long_run,
        "device_status": "ok" if not any(status) else status,
        "distinct_experts_per_step": float(np.mean(U)),
        "replicated_tokens": replicated,
        "prefill": prefill,
        "config1_gemv": gemv1,
        "dense_gemm": dense,
        "sweeps": sweeps,
        "models": models,
    }
    if world > 1:
        got = gather_fn(dist, world)((float(np.mean(uniq)), float(np.mean(pairs_local)),
                                      kernel_ms, [float(v) for v in stage_avg]))
        line["per_rank_active_experts"] = [g[0] for g in got]
        line["per_rank_pairs"] = [g[1] for g in got]
        line["per_rank_kernel_ms"] = [g[2] for g in got]
        line["per_rank_stage_ms"] = [dict(zip(stage_names, g[3])) for g in got]
    if rank == 0:
        print(json.dumps(line), flush=True)
    bad = parity is not None and not parity.get("pass", True)
    # no rank frees its exchange buffers while another may still write to them
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    for lay in layers:
        lay.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if bad:
        print("PARITY FAILED: " + json.dumps(parity), file=sys.stderr, flush=True)
        sys.exit(3)


def parity_block(got, ref, ids, ids_ref, against, n_tok):
    err = float(np.abs(got - ref).max())
    rel = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
    ids_equal = bool(np.array_equal(ids, ids_ref))
    return {"against": against, "tokens": n_tok, "max_abs": err, "rel_l2": rel,
            "ids_equal": ids_equal, "tolerance": {"max_abs": 2e-3, "rel_l2": 1e-3},
            "pass": err <= 2e-3 and rel <= 1e-3 and ids_equal}


def oracle_parity(x_host, out0, ids0, d, F, NE, K, n_tok):
    """rank 0's first tokens of layer 0 (seed 0) against the CPU oracle on
    the same layer, generated on the host by the same seeded generator"""
    from oracle import oracle as orc
    n = min(n_tok, x_host.shape[0])
    L = orc.make_layer(0, d, F, NE, K, orc.Q8_0)
    ref, ids_ref, _, _ = orc.moe_ffn(L, x_host[:n])
    return parity_block(out0[:n], ref, ids0[:n], ids_ref, "oracle (CPU restatement of the "
                        "reference) on the same seeded layer and tokens", n)


def run_prefill(moe, torch, args, layers, rank, world, d, F, NE, K, stream, torch_stream, dist):
    """Prefill leg: P tokens per GPU per layer forward (the grouped tcgen05
    GEMM path), rotated over the same layers, CUDA events (max over ranks).
    N > 1: token-sharded, the token rows and result rows routed with NCCL
    point-to-point transfers around each rank's GEMMs (not capturable: the
    transfer sizes are read on the host), so eager launches."""
    P = args.prefill_tokens
    NL = len(layers)
    shard = moe.EP_SHARDED if world > 1 else 0
    x = synth_tokens(moe, torch, P, d, 0, 6, rank * P, stream)
    out = torch.empty(P * d, dtype=torch.float32, device="cuda")

    def fwd(i, flags=0):
        layers[i % NL].forward_device(x.data_ptr(), out.data_ptr(), P, shard | flags, stream)

    for i in range(max(3, NL)):
        fwd(i)
    torch.cuda.synchronize()
    steps = max(NL, args.prefill_steps)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(torch_stream)
    for i in range(steps):
        fwd(i)
    ev1.record(torch_stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(dist, ev0.elapsed_time(ev1)) / steps
    stage = np.zeros(5)
    pairs = []
    for l in range(NL):
        fwd(l, moe.PROFILE)
        counts = layers[l].routing(P, world)[2]
        first = layers[l].first_expert
        pairs.append(int(counts[first:first + layers[l].n_local].sum()))
    torch.cuda.synchronize()
    for lay in layers:
        s, c = lay.stage_ms()
        stage += np.array(s)
    stage /= NL
    res = {
        "tokens_per_gpu": P, "value": world * P / (ms / 1e3), "unit": "tokens/s",
        "ms_per_step": ms, "steps": steps,
        "stage_ms_avg": {n: float(v) for n, v in
                         zip(["router", "routing", "gate_up", "down", "combine"], stage)},
        "parallelism": "single GPU" if world == 1 else
                       f"expert-parallel x{world}, token-sharded: NCCL all-to-all of the token "
                       "rows and of the result rows around each rank's grouped GEMMs "
                       "(stages of rank 0: routing includes the count exchange, gate_up the "
                       "dispatch transfers, combine the return transfers)",
    }
    if world == 1:
        res["roofline"] = gemm_roofline(stage, float(np.mean(pairs)), d, F)
    return res


def zipf_router_bias(n, s=1.1, seed=4):
    """per-expert router offsets -s * ln(rank), ranks 1..n in a seeded
    random order (config 4's Zipf-skewed expert load)"""
    ranks = np.random.default_rng(seed).permutation(n) + 1
    return (-s * np.log(ranks.astype(np.float64))).astype(np.float32)


def sweep_leg(moe, torch, dist, rank, world, torch_stream, shape, token_counts, cpu_tokens=0,
              NL=2):
    """Config 4 (shape "olmoe": the config-0 layer with a Zipf(1.1)-biased
    router) or the config-3 layer (shape "mixtral": d 4096, d_ff 14336, 8
    experts top-2 renormalised, Q4_0; one expert per GPU at 8 GPUs) over a
    list of per-GPU token counts, token-sharded over the N ranks.  Decode
    sizes are timed from CUDA graphs, larger ones eagerly."""
    stream = torch_stream.cuda_stream
    mixtral = shape == "mixtral"
    if mixtral:
        d, F, NE, K, qtype = 4096, 14336, 8, 2, moe.Q4_0
    else:
        d, F, NE, K, qtype = 2048, 1024, 64, 8, moe.Q8_0
    expert_bytes = 3 * F * d // 32 * (18 if qtype == moe.Q4_0 else 34)
    first, n_local = moe.expert_range(rank, world, NE)
    layers, keep = build_layers(moe, NL, 3 if mixtral else 40, d, F, NE, K, qtype, stream,
                                first, n_local,
                                router_bias=None if mixtral else zipf_router_bias(NE),
                                flags=moe.RENORM if mixtral else 0)
    if world > 1:
        gather = gather_fn(dist, world)
        for lay in layers:
            moe.connect_expert_parallel(lay, rank, gather)
    shard = moe.EP_SHARDED if world > 1 else 0
    hbm_peak, tc_peak, peak_kind = measured_peaks()
    rows = []
    for T in token_counts:
        x = synth_tokens(moe, torch, T, d, 4, 5, rank * T, stream)
        out = torch.empty(T * d, dtype=torch.float32, device="cuda")

        def fwd(i, flags=0):
            layers[i % NL].forward_device(x.data_ptr(), out.data_ptr(), T, shard | flags, stream)

        for i in range(max(3, NL)):
            fwd(i)
        torch.cuda.synchronize()
        counts = []
        for l in range(NL):
            fwd(l)
            counts.append(layers[l].routing(T, world)[2])
        torch.cuda.synchronize()
        fused = T <= DECODE_MAX_T and world * T * K <= 2048
        reps = max(2, min(32, int(1e5 / max(T, 64)) // NL))
        if fused or world == 1:
            ms, g, _ = time_graph_steps(torch, dist, torch_stream, fwd, NL, reps * NL, 0)
            del g
        else:
            if dist:
                dist.barrier()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(torch_stream)
            for i in range(reps * NL):
                fwd(i)
            e1.record(torch_stream)
            torch.cuda.synchronize()
            ms = max_over_ranks(dist, e0.elapsed_time(e1))
        ms /= reps * NL
        loc = [c[first:first + n_local] for c in counts]
        uniq = float(np.mean([(c > 0).sum() for c in loc]))
        pairs = float(np.mean([c.sum() for c in loc]))
        row = {"tokens_per_gpu": T, "value": world * T / (ms / 1e3), "unit": "tokens/s",
               "ms_per_step": ms, "steps": reps * NL, "rank0_experts": uniq,
               "rank0_pairs": pairs, "max_pairs_per_expert": int(counts[0].max()),
               "path": "fused decode kernel" if T <= DECODE_MAX_T else "grouped tcgen05 GEMM"}
        if T <= DECODE_MAX_T:
            row["rank0_achieved_gbs"] = (uniq * expert_bytes + NE * d * 4 + 2 * T * d * 4) / (ms / 1e3) / 1e9
            row["rank0_frac_of_hbm"] = row["rank0_achieved_gbs"] / hbm_peak
        elif world == 1:
            fl = 2.0 * pairs * 3 * d * F
            row["rank0_tflops_algorithmic"] = fl / (ms / 1e3) / 1e12
            row["rank0_frac_of_tensor_peak"] = row["rank0_tflops_algorithmic"] / tc_peak
        else:
            row["rank0_pairs_note"] = "pairs of rank 0's own tokens routed to its experts"
            row["path"] = "NCCL all-to-all around the grouped tcgen05 GEMM"
        if dist:
            got = gather_fn(dist, world)((uniq, pairs))
            row["per_rank_experts"] = [g[0] for g in got]
            row["per_rank_pairs"] = [g[1] for g in got]
        rows.append(row)
        del x, out
        torch.cuda.synchronize()
    cpu = None
    if cpu_tokens and rank == 0:
        cpu = cpu_reference_sample(keep[0], d, F, NE, K, qtype, cpu_tokens, renorm=mixtral)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    for lay in layers:
        lay.close()
    del keep
    torch.cuda.empty_cache()
    return {
        "workload": ("config3: Mixtral-8x7B MoE layer, d 4096, 8 experts top-2 renormalised, "
                     "d_ff 14336, Q4_0") if mixtral else
                    ("config4: config-0 layer with a Zipf(1.1)-biased router"),
        "scaling": "weak (tokens per GPU fixed)" if world > 1 else "single GPU",
        "timing": "CUDA events, max over ranks; graphs for decode sizes, eager above",
        "peaks": {"hbm_gbs": hbm_peak, "bf16_tflops": tc_peak, "source": peak_kind},
        "rows": rows, "cpu_reference": cpu}


def gemm_roofline(stage, pairs, d, F):
    """tensor roofline of the prefill grouped GEMM from the stage times;
    pairs = (token, slot) pairs routed to this rank's experts"""
    flops = 2.0 * pairs * 3 * d * F                  # useful: gate, up, down
    gemm_ms = float(stage[2] + stage[3])
    _, tc_peak, peak_kind = measured_peaks()
    useful = flops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else None
    return {
        "bound": "tensor",
        "kernel": "expert_gemm_kernel<Q8_0> gate/up (dual) + down: tcgen05 kind::f16, "
                  "M 128 pairs x N 256 weight rows, three fp16 hi/lo products",
        "achieved": useful, "unit": "TFLOP/s",
        "achieved_executed": 3 * useful if useful else None,
        "peak": tc_peak, "peak_source": peak_kind + " bf16 dense (burst); fp16 runs at the "
                                          "same tensor rate",
        "frac": useful / tc_peak if useful else None,
        "frac_executed": 3 * useful / tc_peak if useful else None,
        "algorithmic_flops_per_step": flops, "avg_launch_ms": gemm_ms,
        "traffic": None,
        "note": "each product is x_hi w_hi + x_lo w_hi + x_hi w_lo, so the tensor cores "
                "execute 3x the algorithmic FLOPs (the precision bar needs ~22-bit "
                "operands); the gate_up stage includes the fp16 hi/lo gather of the tokens",
        "launch_time_source": "CUDA events between the layer's stages, one profiled "
                              "forward per layer"}


def run_config1_gemv(moe, stream, torch_stream, copies=8, reps=48):
    """Config 1: the dense decode GEMV y = W x, W 14336 x 4096 Q4_0 (33.0 MB,
    seed 1, N(0,0.02) before quantization), x 1 x 4096 fp32, through
    moe_gemv_device.  `copies` distinct weight matrices are rotated (264 MB >
    L2).  Timed twice: eager calls enqueued while a spin kernel holds the
    stream (so the CUDA events see back-to-back device time, not host
    launch gaps), and the same calls captured once in a CUDA graph and
    replayed (one activation row is a single kernel launch with no host
    staging, so it can be captured), as a decode step would run it."""
    import torch
    rows, cols, qt = 14336, 4096, moe.Q4_0
    rb = moe.row_bytes(qt, cols)
    tmp = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    ws = []
    for c in range(copies):
        moe.check(moe.lib().moe_synth_gauss(tmp.data_ptr(), 1 + 100 * c, 2, 0, rows * cols, 0.02,
                                            stream))
        w = torch.empty(rows * rb, dtype=torch.uint8, device="cuda")
        moe.check(moe.lib().moe_quantize_device(tmp.data_ptr(), rows, cols, qt, w.data_ptr(),
                                                stream))
        ws.append(w)
    x = torch.empty(cols, dtype=torch.float32, device="cuda")
    moe.check(moe.lib().moe_synth_gauss(x.data_ptr(), 1, 5, 0, cols, 1.0, stream))
    y = torch.empty(rows, dtype=torch.float32, device="cuda")

    def call(c):
        moe.gemv_device(ws[c].data_ptr(), qt, rows, cols, x.data_ptr(), 1, y.data_ptr(), stream)

    for c in range(3 * copies):
        call(c % copies)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(int(1e8))   # ~50 ms: time to enqueue every call behind it
    e0.record(torch_stream)
    for r in range(reps):
        for c in range(copies):
            call(c)
    e1.record(torch_stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=torch_stream):
        for r in range(6):
            for c in range(copies):
                call(c)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    g0 = torch.cuda.Event(enable_timing=True)
    g1 = torch.cuda.Event(enable_timing=True)
    g0.record(torch_stream)
    for _ in range(reps // 6):
        graph.replay()
    g1.record(torch_stream)
    torch.cuda.synchronize()
    us_graph = g0.elapsed_time(g1) * 1e3 / ((reps // 6) * 6 * copies)
    del graph
    nbytes = rows * rb + cols * 4 + rows * 4
    hbm_peak, _, peak_kind = measured_peaks()
    gbs = nbytes / (us / 1e6) / 1e9
    return {"workload": "config1: dense decode GEMV, W 14336 x 4096 Q4_0, x 1 x 4096 fp32",
            "us_per_gemv": us, "value": 1e6 / us, "unit": "GEMV/s",
            "algorithmic_bytes": nbytes, "achieved_gbs": gbs, "peak_gbs": hbm_peak,
            "frac": gbs / hbm_peak, "peak_source": peak_kind,
            "us_per_gemv_graph": us_graph,
            "frac_graph": nbytes / (us_graph / 1e6) / 1e9 / hbm_peak,
            "launches_per_gemv": 1,
            "timing": f"CUDA events around {reps * copies} back-to-back eager calls over {copies} "
                      "distinct weight matrices (264 MB > L2), enqueued behind a spin kernel; "
                      "_graph: the same calls replayed from a CUDA graph"}


def run_dense_gemm(moe, stream, torch_stream, m=512, reps=20):
    """The dense quantized projections of a prefill through moe_gemv_device
    with m = 512 activation rows (the tcgen05 GEMM with the matrix as one
    expert): config 2's lm_head (50304 x 2048 Q8_0) and an attention
    projection (2048 x 2048 Q8_0); seeded N(0, 0.02) weights, N(0, 1) rows.
    CUDA events around `reps` back-to-back calls; tensor roofline on the
    useful FLOPs (2 m rows cols)."""
    import torch
    _, tc_peak, peak_kind = measured_peaks()
    out = []
    for name, rows, cols in (("lm_head", 50304, 2048), ("attn_proj", 2048, 2048)):
        qt = moe.Q8_0
        tmp = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
        moe.check(moe.lib().moe_synth_gauss(tmp.data_ptr(), 2, 7, 0, rows * cols, 0.02, stream))
        w = torch.empty(rows * moe.row_bytes(qt, cols), dtype=torch.uint8, device="cuda")
        moe.check(moe.lib().moe_quantize_device(tmp.data_ptr(), rows, cols, qt, w.data_ptr(),
                                                stream))
        del tmp
        x = torch.empty(m * cols, dtype=torch.float32, device="cuda")
        moe.check(moe.lib().moe_synth_gauss(x.data_ptr(), 2, 8, 0, m * cols, 1.0, stream))
        y = torch.empty(m * rows, dtype=torch.float32, device="cuda")

        def call():
            moe.gemv_device(w.data_ptr(), qt, rows, cols, x.data_ptr(), m, y.data_ptr(), stream)

        for _ in range(3):
            call()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(torch_stream)
        for _ in range(reps):
            call()
        e1.record(torch_stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        tf = 2.0 * m * rows * cols / (ms / 1e3) / 1e12
        out.append({"workload": f"{name}: {rows} x {cols} Q8_0, m = {m}", "ms": ms,
                    "tflops_algorithmic": tf, "frac_of_tensor_peak": tf / tc_peak,
                    "tflops_executed": 3 * tf, "peak_source": peak_kind + " bf16 (burst)",
                    "weight_gbs": rows * moe.row_bytes(qt, cols) / (ms / 1e3) / 1e9,
                    "launches_per_call": 2})
        del w, x, y
    return out


def run_e2e(moe, args, layers, keep, T, d, F, NE, K, qtype, rank, dist):
    """Same metric through moe_ffn_forward (tensor_t drop-in, host buffers):
    every step copies the tokens host->device and the output device->host."""
    import torch
    import ctypes as C
    nl = min(len(keep), 2)
    hosts = []
    for l in range(nl):
        wr, mats = keep[l]
        hw = wr.cpu().numpy()
        hm = [m.cpu().numpy() for m in mats]
        ts = [moe.tensor(hw, moe.F32, (NE, d)), moe.tensor(hm[0], qtype, (NE, F, d)),
              moe.tensor(hm[1], qtype, (NE, F, d)), moe.tensor(hm[2], qtype, (NE, d, F))]
        for t in ts:
            moe.check(moe.lib().moe_register_weights(C.byref(t)))
        hosts.append(ts)
    xin_p = moe.lib().moe_host_alloc(T * d * 4)
    xout_p = moe.lib().moe_host_alloc(T * d * 4)
    xin = np.ctypeslib.as_array((C.c_float * (T * d)).from_address(xin_p))
    xout = np.ctypeslib.as_array((C.c_float * (T * d)).from_address(xout_p))
    rng = np.random.default_rng(rank)
    xin[:] = rng.standard_normal(T * d).astype(np.float32)
    ti = moe.MoeTensor()
    ti.data = xin_p
    ti.type = moe.F32
    ti.ndim = 2
    ti.dim[0], ti.dim[1] = T, d
    ti.totlen = ti.maxcap = T * d
    to = moe.MoeTensor()
    to.data = xout_p
    to.type = moe.F32
    to.ndim = 2
    to.dim[0], to.dim[1] = T, d
    to.totlen = to.maxcap = T * d

    def call(i):
        h = hosts[i % nl]
        moe.check(moe.lib().moe_ffn_forward(C.byref(ti), C.byref(to), C.byref(h[0]),
                                            C.byref(h[1]), C.byref(h[2]), C.byref(h[3]), K, 0))

    for i in range(max(args.warmup, 2)):
        call(i)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.steps):
        call(i)
    sec = time.perf_counter() - t0
    if dist:
        t = torch.tensor([sec], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        sec = float(t.item())
    world = dist.get_world_size() if dist else 1
    for h in hosts:
        for t in h:
            moe.lib().moe_unregister_weights(C.byref(t))
    moe.lib().moe_host_free(xin_p)
    moe.lib().moe_host_free(xout_p)
    return {"value": world * T * args.steps / sec, "unit": "tokens/s",
            "h2d_bytes_per_step": T * d * 4, "d2h_bytes_per_step": T * d * 4,
            "api": "moe_ffn_forward (tensor_t drop-in; tokens and output in pinned host buffers from moe_host_alloc, host<->device copies inside the call)",
            "timer": "host wall clock around synchronous calls"}


def physical_cores():
    seen = set()
    n = os.cpu_count() or 1
    for c in range(n):
        try:
            with open(f"/sys/devices/system/cpu/cpu{c}/topology/core_id") as f:
                core = f.read().strip()
            pkg = "0"
            p = f"/sys/devices/system/cpu/cpu{c}/topology/physical_package_id"
            if os.path.exists(p):
                with open(p) as f:
                    pkg = f.read().strip()
            seen.add((pkg, core))
        except OSError:
            return n
    return len(seen) or n


def ref_variant():
    flags = ""
    try:
        with open("/proc/cpuinfo") as f:
            flags = f.read()
    except OSError:
        pass
    return "avx512" if " avx512f" in flags else "avx2"


def run_e2e_ep(moe, args, layers, x_host, T, d, stream, dist):
    """Expert-parallel e2e (token-sharded): per step, this rank's tokens come
    from pinned host memory and its output goes back to pinned host memory
    around the layer call (moe_layer_forward); host wall clock per rank, max
    over ranks; value = every rank's tokens."""
    import torch
    nl = len(layers)
    world = dist.get_world_size()
    xin = torch.from_numpy(x_host.reshape(-1).copy()).pin_memory()
    xout = torch.empty(T * d, dtype=torch.float32).pin_memory()
    xd = torch.empty(T * d, dtype=torch.float32, device="cuda")
    od = torch.empty(T * d, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream()

    def call(i):
        xd.copy_(xin, non_blocking=True)
        layers[i % nl].forward_device(xd.data_ptr(), od.data_ptr(), T, moe.EP_SHARDED,
                                      s.cuda_stream)
        xout.copy_(od, non_blocking=True)
        s.synchronize()

    for i in range(max(args.warmup, 2)):
        call(i)
    dist.barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        call(i)
    sec = max_over_ranks(dist, time.perf_counter() - t0)
    return {"value": world * T * args.steps / sec, "unit": "tokens/s",
            "h2d_bytes_per_step": T * d * 4, "d2h_bytes_per_step": T * d * 4,
            "api": "moe_layer_forward with MOE_EP_SHARDED (pinned host -> device copy of this "
                   "rank's tokens and device -> pinned host copy of their output inside the "
                   "step; bytes per GPU)",
            "timer": "host wall clock per rank, max over ranks"}


def cpu_baseline(layer0, x_host, out0, ids0, T, d, F, NE, K, qtype, reps=3):
    """The reference's own CPU path (oracle/_ref, compiled from its sources)
    on the SAME bytes and tokens as the GPU run: the AVX-512 build (what the
    reference's own Makefile selects on this host, -march=native) and the
    AVX2 build, median of `reps` calls after a warm-up.  Its output is the
    parity check of the measured layer: the GPU output of the same layer on
    the same tokens must be within the tolerance, with the same expert ids."""
    from oracle import oracle as orc
    wr, mats = layer0
    arrays = dict(x=x_host, router_w=wr.view(NE, d).cpu().numpy(), gate=mats[0].cpu().numpy(),
                  up=mats[1].cpu().numpy(), down=mats[2].cpu().numpy(), qtype=qtype, d_ff=F,
                  top_k=K, renorm=0)
    res, parity = {}, None
    for variant in ("avx512", "avx2"):
        if not orc.ref_available(variant) or (variant == "avx512" and ref_variant() != "avx512"):
            continue
        r = orc.ref_call("bench", variant, reps=reps, **arrays)
        sec = float(np.median(r["seconds"]))
        res[variant] = {"value": T / sec, "seconds_per_call": sec}
        if parity is None:
            parity = parity_block(out0, r["out"], ids0, r["ids"],
                                  f"the reference itself (oracle/_ref libref_{variant}.so) on "
                                  "identical bytes and tokens", T)
    if not res:
        return ({"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference",
                 "sample": "oracle/_ref not built"}, None)
    main = "avx512" if "avx512" in res else "avx2"
    return ({"value": res[main]["value"], "unit": "tokens/s", "cores": 1, "kind": "reference",
             "variant": main, "builds": res, "host_physical_cores": physical_cores(),
             "sample": f"all {T} config-0 tokens of layer 0 through ref_moe_ffn (reference "
                       "sources, -march=x86-64-v4 / -v3), median of "
                       f"{reps} calls after 1 warm-up, identical bytes to the GPU run; the "
                       "reference runs these expert GEMVs on one thread (below its 16 MFLOP "
                       "threading threshold, thread_pool.c:25,178-185) while its pool spins on "
                       "every physical core"}, parity)


def cpu_reference_sample(layer0, d, F, NE, K, qtype, n_tok, renorm, reps=2):
    """the reference on a few tokens of a layer whose expert GEMVs are above
    its threading threshold (config 3: 117 MFLOP per GEMV), so its thread
    pool runs on every physical core"""
    from oracle import oracle as orc
    variant = ref_variant()
    if not orc.ref_available(variant):
        return None
    wr, mats = layer0
    import torch
    x = torch.randn(n_tok, d, generator=torch.Generator().manual_seed(3)).numpy()
    r = orc.ref_call("bench", variant, reps=reps, x=x, router_w=wr.view(NE, d).cpu().numpy(),
                     gate=mats[0].cpu().numpy(), up=mats[1].cpu().numpy(),
                     down=mats[2].cpu().numpy(), qtype=qtype, d_ff=F, top_k=K,
                     renorm=int(renorm), timeout=1200)
    sec = float(np.median(r["seconds"]))
    return {"value": n_tok / sec, "unit": "tokens/s", "cores": physical_cores(),
            "kind": "reference", "variant": variant,
            "sample": f"{n_tok} tokens through ref_moe_ffn on the config-3 layer, median of "
                      f"{reps} calls after 1 warm-up; above the 16 MFLOP threshold the "
                      "reference splits each GEMV over its thread pool (one thread per "
                      "physical core)"}


# --------------------------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    """The reference's own CPU path (oracle/_ref: its sources compiled as its
    Makefile does, -march=native selects AVX-512 on this host) on the same
    config, metric and unit as our arm: config 0, all T tokens per step."""
    if rank != 0:
        return
    from oracle import oracle as orc
    variant = ref_variant()
    if not orc.ref_available(variant):
        print(json.dumps({"impl": "reference", "unavailable":
                          f"oracle/_ref/libref_{variant}.so not built"}), flush=True)
        return
    d, F, NE, K = 2048, 1024, 64, 8
    L = orc.make_layer(0, d, F, NE, K, orc.Q8_0)
    x = orc.make_tokens(0, args.tokens, d)
    r = orc.ref_call("bench", variant, timeout=3600, x=x, router_w=L["router_w"],
                     gate=L["gate"], up=L["up"], down=L["down"], qtype=orc.Q8_0, d_ff=F,
                     top_k=K, renorm=0, reps=args.steps + args.warmup)
    secs = np.array(r["seconds"])[args.warmup:]
    tot = float(secs.sum())
    val = args.tokens * len(secs) / tot
    avx2 = None
    if variant == "avx512" and orc.ref_available("avx2"):
        r2 = orc.ref_call("bench", "avx2", timeout=3600, x=x, router_w=L["router_w"],
                          gate=L["gate"], up=L["up"], down=L["down"], qtype=orc.Q8_0, d_ff=F,
                          top_k=K, renorm=0, reps=3)
        avx2 = {"value": args.tokens / float(np.median(r2["seconds"])), "unit": "tokens/s",
                "sample": "median of 3 calls after 1 warm-up"}
    cpu = {"value": val, "unit": "tokens/s", "cores": 1, "kind": "reference",
           "variant": variant, "host_physical_cores": physical_cores(),
           "sample": f"all {args.tokens} config-0 tokens per step through ref_moe_ffn "
                     "(single-threaded by the reference's 16 MFLOP threshold)",
           "avx2_build": avx2}
    print(json.dumps({
        "impl": "reference", "metric": "MoE-layer tokens/s (OLMoE config 0, T=%d)" % args.tokens,
        "value": val, "unit": "tokens/s", "n_gpus": world, "steps": len(secs),
        "warmup": args.warmup, "ms_per_step": tot / len(secs) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32 activations x Q8_0 weights",
        "data": "synthetic (seeded N(0,0.02) weights -> Q8_0, N(0,1) tokens)",
        "config": {"workload": "config0: OLMoE-1B-7B MoE FFN layer, d 2048, 64 experts top-8, "
                               "d_ff 1024 SwiGLU, Q8_0, T=%d tokens" % args.tokens,
                   "tokens_per_step": args.tokens},
        "cpu_baseline": cpu,
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)


# --------------------------------------------------------------------------- whole model
# configs 2 and 3: the transformer of olmoe.c / llama.c on the device around
# the MoE layers (moe_model_*), greedy prefill + decode
MODEL_CONFIGS = {
    "config2": dict(arch="olmoe", layers=16, d=2048, heads=16, kv_heads=16, n_exp=64, top_k=8,
                    d_ff=1024, vocab=50304, q="Q8_0", seed=2, prompt=512, decode=128,
                    context=4096, theta=1e4, ref_layers=16, ref_tokens=8, ref_decode=2,
                    name="OLMoE-1B-7B architecture, 16 layers, d 2048, 16 heads, 64 experts "
                         "top-8, d_ff 1024, vocab 50304, Q8_0"),
    "config3": dict(arch="mixtral", layers=32, d=4096, heads=32, kv_heads=8, n_exp=8, top_k=2,
                    d_ff=14336, vocab=32000, q="Q4_0", seed=3, prompt=2048, decode=64,
                    context=4096, theta=1e6, ref_layers=2, ref_tokens=4, ref_decode=1,
                    name="Mixtral-8x7B architecture, 32 layers, d 4096, 32/8 heads, 8 experts "
                         "top-2 (renormalised), d_ff 14336, vocab 32000, Q4_0"),
}


def model_plan(gg, c, layers):
    if c["arch"] == "olmoe":
        return gg.olmoe_plan(layers, c["d"], c["heads"], c["n_exp"], c["top_k"], c["d_ff"],
                             c["vocab"], c["context"], c["theta"])
    return gg.mixtral_plan(layers, c["d"], c["heads"], c["kv_heads"], c["n_exp"], c["top_k"],
                           c["d_ff"], c["vocab"], c["context"], c["theta"])


def synth_model(moe, torch, gg, c, stream):
    """every tensor of the config's file plan generated on the device: matrices
    N(0, 0.02) from generator stream (seed, tag = position in the file) then
    quantized with the reference quantizer's rounding, routers N(0, 0.02)
    fp32, RMSNorm weights ones.  name -> (torch tensor, dtype, dims)"""
    qt = getattr(moe, c["q"])
    _, ts = model_plan(gg, c, c["layers"])
    out = {}
    big = max(int(np.prod(dims)) for _, dims, kind in ts if kind == "mat")
    tmp = torch.empty(big, dtype=torch.float32, device="cuda")
    for tag, (name, dims, kind) in enumerate(ts, start=1):
        n = int(np.prod(dims))
        if kind == "norm":
            out[name] = (torch.ones(n, dtype=torch.float32, device="cuda"), moe.F32, dims)
        elif kind == "router":
            r = torch.empty(n, dtype=torch.float32, device="cuda")
            moe.check(moe.lib().moe_synth_gauss(r.data_ptr(), c["seed"], tag, 0, n, 0.02, stream))
            out[name] = (r, moe.F32, dims)
        else:
            cols = dims[-1]
            rows = n // cols
            moe.check(moe.lib().moe_synth_gauss(tmp.data_ptr(), c["seed"], tag, 0, n, 0.02,
                                                stream))
            q = torch.empty(rows * moe.row_bytes(qt, cols), dtype=torch.uint8, device="cuda")
            moe.check(moe.lib().moe_quantize_device(tmp.data_ptr(), rows, cols, qt, q.data_ptr(),
                                                    stream))
            out[name] = (q, qt, dims)
    torch.cuda.synchronize()
    del tmp
    return out


def model_kv(c, layers):
    a = "olmoe" if c["arch"] == "olmoe" else "llama"
    kv = {"general.architecture": a, "vocab": c["vocab"],
          f"{a}.block_count": layers, f"{a}.embedding_length": c["d"],
          f"{a}.attention.head_count": c["heads"], f"{a}.context_length": c["context"],
          f"{a}.expert_count": c["n_exp"], f"{a}.expert_used_count": c["top_k"],
          f"{a}.feed_forward_length": c["d_ff"], f"{a}.rope.freq_base": c["theta"]}
    if a == "llama":
        kv[f"{a}.attention.head_count_kv"] = c["kv_heads"]
    return kv


def model_decode_bytes(c, at):
    """algorithmic HBM bytes of one decode token with `at` cache rows: every
    layer's attention matrices, router and top_k experts (at most top_k
    distinct), the K and V rows read, lm_head and one embedding row"""
    moe = load_package()
    qt = getattr(moe, c["q"])
    d, hl = c["d"], c["d"] // c["heads"]
    nq, nk = c["heads"] * hl, c["kv_heads"] * hl
    attn = (nq + 2 * nk) * moe.row_bytes(qt, d) + d * moe.row_bytes(qt, nq)
    expert = 2 * c["d_ff"] * moe.row_bytes(qt, d) + d * moe.row_bytes(qt, c["d_ff"])
    kv = 2 * at * nk * 4
    per_layer = attn + c["n_exp"] * d * 4 + c["top_k"] * expert + kv
    return c["layers"] * per_layer + c["vocab"] * moe.row_bytes(qt, d) + moe.row_bytes(qt, d)


def model_prefill_flops(c, T):
    """algorithmic FLOPs of a T-token prefill: 2 x (attention matrices +
    router + top_k experts) per token, causal attention scores and values
    (2 x 2 x T^2/2 x heads x head_len), lm_head of the last row"""
    d, hl = c["d"], c["d"] // c["heads"]
    nq, nk = c["heads"] * hl, c["kv_heads"] * hl
    per_tok = 2 * ((nq + 2 * nk) * d + d * nq + c["n_exp"] * d + c["top_k"] * 3 * c["d_ff"] * d)
    attn = 2 * 2 * (T * T / 2) * nq
    return c["layers"] * (T * per_tok + attn) + 2 * c["vocab"] * d


def model_reference_sample(moe, torch, gg, c, tensors, model_small):
    """The reference's own model code (oracle/_ref/libref_model.so: olmoe.c /
    llama.c) on a GGUF file written from the same device bytes, truncated to
    ref_layers layers: a ref_tokens-token prefill and ref_decode greedy
    steps, timed on the host cores, and this library's model of the same
    layers on the same tokens checked against it."""
    from oracle import oracle as orc
    if not orc.ref_available("model") or ref_variant() != "avx512":
        return None, {"pass": None, "skipped": "oracle/_ref/libref_model.so not built or no "
                                               "AVX-512 host"}
    import tempfile
    L = c["ref_layers"]
    plan = model_plan(gg, c, L)
    def fetch(name):
        t = tensors[name][0]
        return t.cpu().numpy()

    td = tempfile.mkdtemp(prefix="moe_model_")
    path = os.path.join(td, "sample.gguf")
    t0 = time.perf_counter()
    gg.write_plan_from(path, plan, getattr(moe, c["q"]), fetch)
    write_s = time.perf_counter() - t0
    rng = np.random.default_rng(c["seed"] + 100)
    toks = rng.integers(0, c["vocab"], c["ref_tokens"]).astype(np.int32)
    try:
        r = orc.ref_call("model", "model", timeout=1800, path=path, tokens=toks,
                         n_decode=c["ref_decode"], d_model=c["d"], vocab=c["vocab"])
    finally:
        os.unlink(path)
        os.rmdir(td)
    # this library, same layers, same tokens, teacher-forced with the
    # reference's picks
    model_small.reset()
    rows = model_small.prefill(toks)
    errs, rels = [], []

    def cmp(got, want):
        got = np.asarray(got, np.float64)
        want = np.asarray(want, np.float64)
        errs.append(float(np.abs(got - want).max()))
        rels.append(float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)))

    cmp(rows, r["rows"])
    cmp(model_small.logits(len(toks) - 1), r["logits"][0])
    for i, t in enumerate(r["tokens"]):
        cmp(model_small.decode(int(t), len(toks) + i), r["drows"][i])
        cmp(model_small.logits(0), r["logits"][i + 1])
    picks_ok = True
    model_small.reset()
    picks = model_small.generate(toks, c["ref_decode"])
    for i, t in enumerate(r["tokens"]):
        top2 = np.sort(r["logits"][i])[-2:]
        if top2[1] - top2[0] < 1e-3:
            break
        picks_ok = picks_ok and int(picks[i]) == int(t)
    model_small.reset()
    scale = L / c["layers"]
    pf = float(r["prefill_seconds"])
    dc = float(r["decode_seconds"])
    cpu = {"prefill_tok_s": len(toks) / pf * scale, "decode_tok_s": c["ref_decode"] / dc * scale,
           "unit": "tokens/s", "cores": physical_cores(), "kind": "reference",
           "sample": f"the reference's olmoe.c/llama.c forward (AVX-512 build, its thread pool "
                     f"on every core) on {L} of {c['layers']} layers of the same weights: a "
                     f"{len(toks)}-token prefill ({pf:.2f} s) and {c['ref_decode']} greedy "
                     f"decode steps with lm_head ({dc:.2f} s); tokens/s scaled by "
                     f"{L}/{c['layers']} layers",
           "gguf_write_s": write_s}
    parity = {"pass": bool(max(errs) <= 2e-3 and max(rels) <= 1e-3 and picks_ok),
              "max_abs": max(errs), "rel_l2": max(rels), "greedy_picks_match": picks_ok,
              "against": "the reference's own model code (oracle/_ref/libref_model.so) on a "
                         f"GGUF of the same bytes, {L} layers",
              "checked": f"{len(toks)} prefill rows, {c['ref_decode']} decode rows, "
                         f"{c['ref_decode'] + 1} logit rows, greedy picks",
              "tolerance": "max-abs 2e-3, rel-L2 1e-3"}
    return cpu, parity


def run_model_leg(moe, torch, torch_stream, cfg_name, runs=3, with_ref=True, clocks_dev=0,
                  n_decode=0):
    """One whole-model config on one GPU: weights generated in HBM, the
    model built from them (moe_model_create), then greedy generation of the
    config's decode steps after its prompt, timed by the model's CUDA events
    (prefill with the first pick; decode steps with lm_head and pick) and,
    for e2e, by the host clock around the call (host prompt in, host tokens
    out).  One warm-up generation; `runs` timed ones, median reported."""
    gg = load_gguf_module()
    c = MODEL_CONFIGS[cfg_name]
    stream = torch_stream.cuda_stream
    t0 = time.perf_counter()
    tensors = synth_model(moe, torch, gg, c, stream)
    synth_s = time.perf_counter() - t0

    def get(name):
        t, dt, dims = tensors[name]
        return moe.tensor_at(t.data_ptr(), dt, dims)

    small = None
    if with_ref and c["ref_layers"] < c["layers"]:
        small = moe.Model.build(model_kv(c, c["ref_layers"]), get)
    t0 = time.perf_counter()
    model = moe.Model.build(model_kv(c, c["layers"]), get)
    create_s = time.perf_counter() - t0
    cpu, parity = None, None
    if with_ref:
        cpu, parity = model_reference_sample(moe, torch, gg, c, tensors, small or model)
    if small is not None:
        small.close()
    del tensors
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    prompt = np.random.default_rng(c["seed"]).integers(0, c["vocab"], c["prompt"]).astype(np.int32)
    n = n_decode or c["decode"]
    model.reset()
    model.generate(prompt, n)
    model.reset()
    clocks = ClockSampler(clocks_dev)
    clocks.start()
    pf, dc, wall, made = [], [], [], 0
    for _ in range(runs):
        w0 = time.perf_counter()
        picks = model.generate(prompt, n)
        wall.append(time.perf_counter() - w0)
        made = picks.size
        a, b = model.timing()
        pf.append(a)
        dc.append(b)
        model.reset()
    clk = clocks.stop()
    _, _, dev_bytes = model.info()
    mode = model.mode()
    status = model.status()
    model.close()
    pf_ms, dc_ms, wall_s = float(np.median(pf)), float(np.median(dc)), float(np.median(wall))
    steps = made - 1
    hbm_peak, bf16_peak, peak_kind = measured_peaks()
    at = c["prompt"] + steps / 2
    dbytes = model_decode_bytes(c, at)
    dec_tok_s = steps / (dc_ms / 1e3) if steps else None
    flops = model_prefill_flops(c, c["prompt"])
    return {
        "workload": f"{cfg_name}: {c['name']}; {c['prompt']}-token uniform-random prompt, then "
                    f"{n} greedy decode steps with KV cache (seed {c['seed']})",
        "prefill_tok_s": c["prompt"] / (pf_ms / 1e3), "prefill_ms": pf_ms,
        "decode_tok_s": dec_tok_s, "decode_ms_per_token": dc_ms / max(steps, 1),
        "decode_steps": steps, "unit": "tokens/s",
        "e2e": {"tok_s": (c["prompt"] + steps) / wall_s, "seconds": wall_s,
                "h2d_bytes": int(prompt.nbytes), "d2h_bytes": int(4 * made),
                "what": "moe_model_generate from host token ids to host picks, host clock"},
        "decode_roofline": {"bound": "hbm", "bytes_per_token": dbytes,
                            "achieved_gbs": dbytes * dec_tok_s / 1e9 if dec_tok_s else None,
                            "peak_gbs": hbm_peak, "frac": (dbytes * dec_tok_s / 1e9 / hbm_peak)
                            if dec_tok_s else None, "peak_source": peak_kind,
                            "cache_rows_mean": at},
        "prefill_roofline": {"bound": "tensor", "flops": flops,
                             "achieved_tflops": flops / (pf_ms / 1e3) / 1e12,
                             "peak_tflops": bf16_peak,
                             "frac": flops / (pf_ms / 1e3) / 1e12 / bf16_peak},
        "cpu_baseline": cpu, "parity": parity, "clocks": clk,
        "device_status": "ok" if status == 0 else status,
        "device_bytes": dev_bytes, "synth_s": synth_s, "create_s": create_s,
        "decode_step": mode,
        "timing": f"CUDA events inside moe_model_generate, median of {runs} runs after one "
                  "warm-up; decode steps replay one CUDA graph each",
    }


def load_gguf_module():
    import importlib.util
    p = os.path.join(ROOT, "llm.c_b200", "gguf.py")
    spec = importlib.util.spec_from_file_location("moe_gguf", p)
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=32, help="tokens per GPU per step")
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--prefill-tokens", type=int, default=2048,
                    help="tokens per GPU of the prefill leg (0: skip)")
    ap.add_argument("--prefill-steps", type=int, default=16)
    ap.add_argument("--sweep4", default="1,8,64,512,4096",
                    help="per-GPU token counts of the config-4 leg")
    ap.add_argument("--sweep3", default="1,32,512",
                    help="per-GPU token counts of the config-3 leg")
    ap.add_argument("--parity-tokens", type=int, default=8,
                    help="tokens of rank 0 checked against the oracle at N > 1")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline legs")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e leg")
    ap.add_argument("--no-gemv", action="store_true", help="skip the config-1 GEMV leg")
    ap.add_argument("--no-sweeps", action="store_true", help="skip the config-3/4 legs")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check at N > 1")
    ap.add_argument("--no-replicated", action="store_true",
                    help="skip the replicated-token leg at N > 1")
    ap.add_argument("--no-model", action="store_true",
                    help="skip the whole-model legs (configs 2 and 3)")
    ap.add_argument("--models", default="config2,config3",
                    help="whole-model configs timed at N=1")
    ap.add_argument("--model-decode", type=int, default=0,
                    help="decode steps of the model legs (0: the config's)")
    ap.add_argument("--model-runs", type=int, default=3, help="timed generations per model leg")
    ap.add_argument("--only", choices=["gemv", "dense", "config2", "config3"],
                    help="run one leg alone on one GPU (for profilers) and print its result")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    args.steps = max(args.steps, 1)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
    elif args.only:
        torch, moe, _, torch_stream = init_rank(1, local_rank)
        if args.only in MODEL_CONFIGS:
            res = run_model_leg(moe, torch, torch_stream, args.only, runs=args.model_runs,
                                with_ref=not args.no_cpu, clocks_dev=local_rank,
                                n_decode=args.model_decode)
        else:
            leg = run_config1_gemv if args.only == "gemv" else run_dense_gemm
            res = leg(moe, torch_stream.cuda_stream, torch_stream)
        print(json.dumps({"only": args.only, "result": res}), flush=True)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
