#!/usr/bin/env python3
"""Benchmark of the B200 MoE FFN layer (BASELINE.json metric: MoE-layer
tokens/s and achieved HBM TB/s).

Default workload = BASELINE config 0: one OLMoE-1B-7B-shaped MoE FFN layer
(d_model 2048, 64 experts, top-8 without renormalisation, d_ff 1024 SwiGLU,
Q8_0 experts, fp32 router) on T = 32 tokens.  A step is one layer forward
over the T tokens.  Weights are synthetic (seeded N(0, 0.02) through the
shared generator, quantized to Q8_0 on the device); NL distinct layers are
rotated so that every step streams 428 MB of experts that are not in the
126 MB L2.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--tokens T] [--layers NL] [--prefill-tokens P]

Prints one JSON line (rank 0).  Under torchrun the layer is expert-parallel:
rank r holds experts expert_range(r) of every layer, every rank gets the
same T tokens and ends with the full output (strong scaling); the time is
the max over ranks.  On one GPU the line also carries a "prefill" object:
the same layers on P tokens (default 2048), which runs the tcgen05 grouped
GEMM, with its tensor roofline.
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


# --------------------------------------------------------------------------- ours
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


def run_ours(args, rank, world, local_rank):
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
    stream = torch_stream.cuda_stream
    d, F, NE, K, qtype = 2048, 1024, 64, 8, moe.Q8_0
    T = args.tokens
    NL = args.layers
    # N > 1: expert parallelism, rank r holds experts expert_range(r) of every
    # layer; the tokens are the same on every rank (replicated, as after a
    # replicated attention block) and every rank ends with the full output
    first, n_local = moe.expert_range(rank, world, NE)
    layers, keep = build_layers(moe, NL, 0, d, F, NE, K, qtype, stream, first, n_local)
    if world > 1:
        def gather(obj):
            got = [None] * world
            dist.all_gather_object(got, obj)
            return got
        for lay in layers:
            moe.connect_expert_parallel(lay, rank, gather)
        # batches above 64 tokens sum the ranks' partial outputs (NCCL)
        moe.init_expert_parallel_comm(rank, world, gather)
    # tokens: config-0 input seed 0, tag 5
    x = torch.empty(T * d, dtype=torch.float32, device="cuda")
    moe.check(moe.lib().moe_synth_gauss(x.data_ptr(), 0, 5, 0, T * d, 1.0, stream))
    out = torch.empty(T * d, dtype=torch.float32, device="cuda")

    def step(i, flags=0):
        layers[i % NL].forward_device(x.data_ptr(), out.data_ptr(), T, flags, stream)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    # routing of the layers (distinct experts touched = algorithmic bytes)
    uniq, pairs_local = [], []
    for l in range(NL):
        step(l)
        ids_all = layers[l].routing(T)[0]
        ids = np.unique(ids_all)
        uniq.append(int(((ids >= first) & (ids < first + n_local)).sum()))  # this rank's experts
        pairs_local.append(int(((ids_all >= first) & (ids_all < first + n_local)).sum()))
    torch.cuda.synchronize()

    # The timed steps replay a CUDA graph of the NL rotated layer forwards
    # (one graph launch per NL steps), so host launch overhead is out of the
    # device timing.  Each captured forward records per-stage timestamps
    # (external event records) that reflect the last replay.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=torch_stream, capture_error_mode="relaxed"):
        for l in range(NL):
            step(l, moe.PROFILE)
    graph.replay()
    torch.cuda.synchronize()
    reps = max(1, args.steps // NL)
    args.steps = reps * NL

    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    h0 = time.perf_counter()
    ev0.record(torch_stream)
    for _ in range(reps):
        graph.replay()
    ev1.record(torch_stream)
    host_ms = (time.perf_counter() - h0) * 1e3
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clk = clocks.stop()
    ms_total = ev0.elapsed_time(ev1)
    stage = np.zeros(5)
    nprof = 0
    for lay in layers:
        try:
            s, c = lay.stage_ms()
            stage += np.array(s)
            nprof += c
        except moe.MoeError:
            pass
    if dist:
        t = torch.tensor([ms_total], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    ms_step = ms_total / args.steps
    # every rank ends a step with the output of the same T tokens
    tokens_per_s = T * args.steps / (ms_total / 1e3)

    # ---- e2e: reference-facing tensor_t call with host buffers (H2D + D2H inside)
    if args.no_e2e:
        e2e = None
    elif world == 1:
        e2e = run_e2e(moe, args, layers, keep, T, d, F, NE, K, qtype, rank, dist)
    else:
        e2e = run_e2e_ep(moe, args, layers, T, d, stream, dist)

    # ---- roofline of the dominant kernel: the fused decode-layer kernel, one
    # launch per layer forward (router, routing, gate/up + SwiGLU, down, combine)
    hbm_peak, _, peak_kind = measured_peaks()
    U = np.array([uniq[i % NL] for i in range(args.steps)], float)
    layer_bytes = float(np.mean(U)) * EXPERT_BYTES_Q8 + NE * d * 4 + 2 * T * d * 4
    stage_avg = stage / max(nprof, 1)
    kernel_ms = float(stage_avg.sum())
    achieved = layer_bytes / (kernel_ms / 1e3) / 1e9 if kernel_ms > 0 else None
    roof = {"bound": "hbm",
            "kernel": "moe_decode_kernel<Q8_0, 16 lanes> (whole MoE layer, one launch)",
            "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
            "frac": achieved / hbm_peak if achieved else None, "traffic": None,
            "peak_source": peak_kind,
            "algorithmic_bytes_per_launch": layer_bytes, "avg_launch_ms": kernel_ms,
            "launch_time_source": "%globaltimer stamps of every CTA (earliest start to "
                                  "latest end), averaged over the profiled replays",
            "step_achieved_gbs": layer_bytes / (ms_step / 1e3) / 1e9,
            "stage_ms_avg": {n: float(v) for n, v in
                             zip(["router", "routing", "gate_up", "down", "combine"], stage_avg)}}
    if T > DECODE_MAX_T:
        roof = dict(gemm_roofline(stage_avg, float(np.mean(pairs_local)), d, F),
                    stage_ms_avg=roof["stage_ms_avg"], step_ms=ms_step)
    traffic = os.path.join(ROOT, "profiles", "traffic.json")
    if T <= DECODE_MAX_T and os.path.exists(traffic):
        with open(traffic) as f:
            tj = json.load(f)
        # DRAM bytes of one captured launch, scaled by the routed experts
        per_expert, fixed = tj.get("bytes_per_active_expert"), tj.get("bytes_fixed", 0.0)
        if per_expert and tj.get("kernel") == roof["kernel"]:
            roof["traffic"] = per_expert * float(np.mean(U)) + fixed
            roof["traffic_source"] = "profiles/" + tj.get("source", "traffic.json")

    prefill = None
    if args.prefill_tokens > 0:
        prefill = run_prefill(moe, args, layers, d, F, NE, K, stream, torch_stream, dist)

    gemv1 = None
    if world == 1 and not args.no_gemv:
        gemv1 = run_config1_gemv(moe, stream, torch_stream)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(moe, keep[0], x, T, d, F, NE, K, qtype)

    line = {
        "metric": "MoE-layer tokens/s (OLMoE config 0, T=%d)" % T,
        "value": tokens_per_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32 activations x Q8_0 weights",
        "data": "synthetic (seeded N(0,0.02) weights -> Q8_0, N(0,1) tokens)",
        "config": {"workload": "config0: OLMoE-1B-7B MoE FFN layer, d 2048, 64 experts top-8, "
                               "d_ff 1024 SwiGLU, Q8_0, T=%d tokens" % T,
                   "tokens_per_step": T, "layers_rotated": NL,
                   "l2": f"{NL} distinct layers rotated; each step streams "
                         f"{np.mean(U) * EXPERT_BYTES_Q8 / 1e6:.0f} MB of experts > 126 MB L2",
                   "parallelism": (f"expert-parallel x{world}: {n_local} experts per GPU, the "
                                   "(token, slot) rows exchanged over NVLink inside the fused "
                                   "kernel, every GPU combines the full output")
                                  if world > 1 else "single GPU"},
        "e2e": e2e, "roofline": roof, "cpu_baseline": cpu, "clocks": clk,
        # one fused decode-layer kernel per forward; above 64 tokens: router,
        # top-k + dispatch (one launch up to 256 tokens, two above), gather,
        # two GEMMs and the combine
        "gpu_launches": args.steps * (1 if T <= DECODE_MAX_T else 6 if T <= 256 else 7),
        "host_enqueue_ms": host_ms,
        "timing": "CUDA events on the launching stream around CUDA-graph replays "
                  f"({NL} layer forwards per graph)",
        "distinct_experts_per_step": float(np.mean(U)),
        "prefill": prefill,
        "config1_gemv": gemv1,
    }
    if world > 1:
        got = [None] * world
        dist.all_gather_object(got, (float(np.mean(uniq)), kernel_ms))
        line["per_rank_active_experts"] = [g[0] for g in got]
        line["per_rank_kernel_ms"] = [g[1] for g in got]
    if rank == 0:
        print(json.dumps(line), flush=True)
    # no rank frees its exchange buffers while another may still write to them
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    for lay in layers:
        lay.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


DECODE_MAX_T = 64   # batches above this take the prefill GEMM path


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


def run_prefill(moe, args, layers, d, F, NE, K, stream, torch_stream, dist=None):
    """Prefill leg: P tokens per layer forward (the grouped tcgen05 GEMM
    path), rotated over the same layers; device time with CUDA events (max
    over ranks), the stages from one profiled forward per layer.  Expert
    parallel (N > 1): every rank runs its experts' GEMMs on the same P
    tokens and the partial outputs are summed by the library's NCCL
    all-reduce inside the step."""
    import torch
    P = args.prefill_tokens
    NL = len(layers)
    x = torch.empty(P * d, dtype=torch.float32, device="cuda")
    moe.check(moe.lib().moe_synth_gauss(x.data_ptr(), 0, 6, 0, P * d, 1.0, stream))
    out = torch.empty(P * d, dtype=torch.float32, device="cuda")

    def fwd(i, flags=0):
        layers[i % NL].forward_device(x.data_ptr(), out.data_ptr(), P, flags, stream)

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
    ms = ev0.elapsed_time(ev1) / steps
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    stage = np.zeros(5)
    pairs = []
    for l in range(NL):
        fwd(l, moe.PROFILE)
        ids = layers[l].routing(P)[0]
        first = layers[l].first_expert
        pairs.append(int(((ids >= first) & (ids < first + layers[l].n_local)).sum()))
    torch.cuda.synchronize()
    for lay in layers:
        s, c = lay.stage_ms()
        stage += np.array(s)
    stage /= NL
    return {
        "tokens": P, "value": P / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
        "steps": steps,
        "stage_ms_avg": {n: float(v) for n, v in
                         zip(["router", "routing", "gate_up", "down", "combine"], stage)},
        "roofline": gemm_roofline(stage, float(np.mean(pairs)), d, F),
        "parallelism": "single GPU" if not dist else
                       f"expert-parallel x{dist.get_world_size()}: GEMMs of the local experts, "
                       "partial outputs summed by an NCCL all-reduce in the step (stages and "
                       "roofline of rank 0)",
    }


def zipf_router_bias(n, s=1.1, seed=4):
    """per-expert router offsets -s * ln(rank), ranks 1..n in a seeded
    random order (config 4's Zipf-skewed expert load)"""
    ranks = np.random.default_rng(seed).permutation(n) + 1
    return (-s * np.log(ranks.astype(np.float64))).astype(np.float32)


def run_sweep(args, rank, world, local_rank):
    """Config 4: the config-0 layer with a Zipf(1.1)-biased router over a
    sweep of token counts, expert-parallel over the N ranks (64/N experts
    each).  --sweep-shape mixtral: the config-3 layer instead (d 4096, d_ff
    14336, 8 experts top-2 renormalised, Q4_0, no router offsets; at 8 GPUs
    one expert per GPU).  One JSON line with one entry per T."""
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
    torch_stream = torch.cuda.Stream()
    torch.cuda.set_stream(torch_stream)
    stream = torch_stream.cuda_stream
    mixtral = args.sweep_shape == "mixtral"
    if mixtral:
        d, F, NE, K, qtype = 4096, 14336, 8, 2, moe.Q4_0
    else:
        d, F, NE, K, qtype = 2048, 1024, 64, 8, moe.Q8_0
    expert_bytes = 3 * F * d // 32 * (18 if qtype == moe.Q4_0 else 34)
    NL = 2
    first, n_local = moe.expert_range(rank, world, NE)
    layers, keep = build_layers(moe, NL, 3 if mixtral else 40, d, F, NE, K, qtype, stream,
                                first, n_local,
                                router_bias=None if mixtral else zipf_router_bias(NE),
                                flags=moe.RENORM if mixtral else 0)
    if world > 1:
        def gather(obj):
            got = [None] * world
            dist.all_gather_object(got, obj)
            return got
        for lay in layers:
            moe.connect_expert_parallel(lay, rank, gather)
        moe.init_expert_parallel_comm(rank, world, gather)
    hbm_peak, tc_peak, peak_kind = measured_peaks()
    rows = []
    for T in [int(t) for t in args.sweep.split(",")]:
        x = torch.empty(T * d, dtype=torch.float32, device="cuda")
        moe.check(moe.lib().moe_synth_gauss(x.data_ptr(), 4, 5, 0, T * d, 1.0, stream))
        out = torch.empty(T * d, dtype=torch.float32, device="cuda")

        def fwd(i, flags=0):
            layers[i % NL].forward_device(x.data_ptr(), out.data_ptr(), T, flags, stream)

        for i in range(max(3, NL)):
            fwd(i)
        torch.cuda.synchronize()
        ids = [None] * NL
        for l in range(NL):
            fwd(l)
            ids[l] = layers[l].routing(T)[0]
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=torch_stream, capture_error_mode="relaxed"):
            for l in range(NL):
                fwd(l)
        graph.replay()
        torch.cuda.synchronize()
        reps = max(2, min(64, int(2e5 / max(T, 64)) // NL))
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(torch_stream)
        for _ in range(reps):
            graph.replay()
        e1.record(torch_stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / (reps * NL)
        if dist:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        local = [((a >= first) & (a < first + n_local)) for a in ids]
        uniq = float(np.mean([len(np.unique(a[m])) for a, m in zip(ids, local)]))
        pairs = float(np.mean([m.sum() for m in local]))
        counts = np.bincount(ids[0].reshape(-1), minlength=NE)
        row = {"tokens": T, "value": T / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
               "steps": reps * NL, "rank0_experts": uniq, "rank0_pairs": pairs,
               "max_pairs_per_expert": int(counts.max()),
               "path": "fused decode kernel" if T <= DECODE_MAX_T else "grouped tcgen05 GEMM"}
        if T <= DECODE_MAX_T:
            row["rank0_achieved_gbs"] = (uniq * expert_bytes + NE * d * 4 + 2 * T * d * 4) / (ms / 1e3) / 1e9
            row["rank0_frac_of_hbm"] = row["rank0_achieved_gbs"] / hbm_peak
        else:
            fl = 2.0 * pairs * 3 * d * F
            row["rank0_tflops_algorithmic"] = fl / (ms / 1e3) / 1e12
            row["rank0_frac_of_tensor_peak"] = row["rank0_tflops_algorithmic"] / tc_peak
        if dist:
            got = [None] * world
            dist.all_gather_object(got, (uniq, pairs))
            row["per_rank_experts"] = [g[0] for g in got]
            row["per_rank_pairs"] = [g[1] for g in got]
        rows.append(row)
        graph = None
        del x, out
        torch.cuda.synchronize()
    if rank == 0:
        print(json.dumps({
            "metric": ("MoE-layer tokens/s over a token sweep (config-3 layer: Mixtral-8x7B "
                       "shape, Q4_0, top-2 renormalised)") if mixtral else
                      ("MoE-layer tokens/s over a token sweep (config 4: config-0 layer, "
                       "Zipf(1.1)-biased router)"),
            "n_gpus": world, "unit": "tokens/s", "higher_is_better": True,
            "scaling": "strong",
            "data": "synthetic (seeded N(0,0.02) weights -> %s, N(0,1) tokens%s)" % (
                "Q4_0" if mixtral else "Q8_0", "" if mixtral else ", Zipf(1.1) router offsets"),
            "timing": "CUDA events around CUDA-graph replays of 2 rotated layers, max over ranks; "
                      "whole step (the layer forward) per T",
            "peaks": {"hbm_gbs": hbm_peak, "bf16_tflops": tc_peak, "source": peak_kind},
            "parallelism": f"expert-parallel x{world}" if world > 1 else "single GPU",
            "sweep": rows}), flush=True)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    for lay in layers:
        lay.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


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


def run_e2e_ep(moe, args, layers, T, d, stream, dist):
    """Expert-parallel e2e: per step, this rank's tokens come from pinned host
    memory and its output goes back to pinned host memory around the layer
    call (moe_layer_forward); wall clock per rank, max over ranks."""
    import torch
    nl = len(layers)
    xin = torch.randn(T * d, dtype=torch.float32, generator=torch.Generator().manual_seed(0))
    xin = xin.pin_memory()
    xout = torch.empty(T * d, dtype=torch.float32).pin_memory()
    xd = torch.empty(T * d, dtype=torch.float32, device="cuda")
    od = torch.empty(T * d, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream()

    def call(i):
        xd.copy_(xin, non_blocking=True)
        layers[i % nl].forward_device(xd.data_ptr(), od.data_ptr(), T, 0, s.cuda_stream)
        xout.copy_(od, non_blocking=True)
        s.synchronize()

    for i in range(max(args.warmup, 2)):
        call(i)
    dist.barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        call(i)
    sec = time.perf_counter() - t0
    t = torch.tensor([sec], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    sec = float(t.item())
    return {"value": T * args.steps / sec, "unit": "tokens/s",
            "h2d_bytes_per_step": T * d * 4, "d2h_bytes_per_step": T * d * 4,
            "api": "moe_layer_forward (expert-parallel; pinned host -> device copy of the "
                   "tokens and device -> pinned host copy of the output inside the step)",
            "timer": "host wall clock per rank, max over ranks"}


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


def cpu_baseline(moe, layer0, x_dev, T, d, F, NE, K, qtype, sample_tokens=8, reps=3):
    """The reference's own CPU path (oracle/_ref, compiled from its sources)
    on the SAME bytes as the GPU run, on a bounded sample of tokens."""
    from oracle import oracle as orc
    variant = ref_variant()
    if not orc.ref_available(variant):
        return {"value": None, "unit": "tokens/s", "cores": 0, "kind": "reference",
                "sample": f"oracle/_ref/libref_{variant}.so not built"}
    wr, mats = layer0
    xs = x_dev.view(T, d)[:sample_tokens].cpu().numpy()
    r = orc.ref_call("bench", variant, x=xs, router_w=wr.view(NE, d).cpu().numpy(),
                     gate=mats[0].cpu().numpy(), up=mats[1].cpu().numpy(),
                     down=mats[2].cpu().numpy(), qtype=qtype, d_ff=F, top_k=K, renorm=0,
                     reps=reps)
    sec = float(np.median(r["seconds"]))
    return {"value": sample_tokens / sec, "unit": "tokens/s", "cores": 1, "kind": "reference",
            "variant": variant, "host_physical_cores": physical_cores(),
            "sample": f"{sample_tokens} of the {T} config-0 tokens through ref_moe_ffn "
                      f"(reference sources, -march=x86-64-{'v4' if variant == 'avx512' else 'v3'}), "
                      f"median of {reps} calls after 1 warm-up, identical bytes to the GPU run; "
                      "the reference runs these expert GEMVs on one thread (below its 16 MFLOP "
                      "threading threshold) while its pool spins on every physical core"}


# --------------------------------------------------------------------------- reference arm
def run_reference(args, rank, world):
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
    S = min(8, args.tokens)
    r = orc.ref_call("bench", variant, timeout=3600, x=x[:S], router_w=L["router_w"],
                     gate=L["gate"], up=L["up"], down=L["down"], qtype=orc.Q8_0, d_ff=F,
                     top_k=K, renorm=0, reps=args.steps + args.warmup)
    secs = np.array(r["seconds"])[args.warmup:]
    tot = float(secs.sum())
    val = S * len(secs) / tot
    cpu = {"value": val, "unit": "tokens/s", "cores": 1, "kind": "reference",
           "variant": variant, "host_physical_cores": physical_cores(),
           "sample": f"{S} of the {args.tokens} config-0 tokens per step through ref_moe_ffn"}
    print(json.dumps({
        "impl": "reference", "metric": "MoE-layer tokens/s (OLMoE config 0, T=%d)" % args.tokens,
        "value": val, "unit": "tokens/s", "n_gpus": world, "steps": len(secs),
        "warmup": args.warmup, "ms_per_step": tot / len(secs) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32 activations x Q8_0 weights",
        "data": "synthetic (seeded N(0,0.02) weights -> Q8_0, N(0,1) tokens)",
        "config": {"workload": "config0: OLMoE-1B-7B MoE FFN layer on the reference CPU path"},
        "cpu_baseline": cpu,
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=32)
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--prefill-tokens", type=int, default=2048,
                    help="tokens of the one-GPU prefill leg (0: skip)")
    ap.add_argument("--prefill-steps", type=int, default=16)
    ap.add_argument("--sweep", default="",
                    help="comma-separated token counts: run config 4 (Zipf router) instead")
    ap.add_argument("--sweep-shape", choices=["olmoe", "mixtral"], default="olmoe")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e leg")
    ap.add_argument("--no-gemv", action="store_true", help="skip the config-1 GEMV leg")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
    elif args.sweep:
        run_sweep(args, rank, world, local_rank)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
