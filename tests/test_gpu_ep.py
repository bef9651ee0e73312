"""Expert parallelism on 2+ GPUs: every rank owns a contiguous range of
experts (expert_range).  Two ways to split the work, both checked here on
every visible GPU (up to 8 ranks):

* replicated tokens (default): every rank passes the same T tokens and ends
  with the full output.  Decode batches run the fused decode kernel, which
  writes the rows of its experts into every rank's exchange buffer over
  NVLink; larger batches run the grouped GEMMs on the local experts and sum
  the ranks' partial outputs with the library's NCCL all-reduce.  Every
  rank's output must be identical across ranks, identical to one GPU
  (decode) or within fp32 reassociation of it (larger batches), and within
  the tolerance of the CPU oracle.
* token-sharded (MOE_EP_SHARDED): rank r passes rows [r*T, (r+1)*T) of one
  global batch and gets their outputs.  Decode batches run the fused kernel
  (tokens and ids gathered over NVLink, each row stored into the owning
  rank's buffer); larger batches route the token rows and the result rows
  with NCCL point-to-point transfers around the grouped GEMMs.  Each rank's
  output must equal one GPU's forward of the same rows (bit for bit for the
  fused kernel) and the oracle within tolerance.

Skipped where fewer than two GPUs are visible.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_package

pytestmark = pytest.mark.gpu

MAX_ABS, REL_L2 = 2e-3, 1e-3


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def local_experts(moe, L, name, first, nl, keep):
    """device copies of this rank's experts of one matrix (0 for the others)"""
    ptrs = []
    for e in range(L["n_experts"]):
        if first <= e < first + nl:
            b = moe.DeviceBuffer.from_numpy(np.ascontiguousarray(L[name][e]))
            keep.append(b)
            ptrs.append(b.ptr)
        else:
            ptrs.append(0)
    return ptrs


def _rank_main(rank, world, port, shape, token_counts, sharded, results):
    """sharded: a bool for every forward, or a list with one per forward"""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    moe = load_package()
    try:
        from oracle import oracle as orc
        d, F, NE, K, qt, seed = shape
        L = orc.make_layer(seed, d, F, NE, K, qt)
        moe.init(rank)
        first, nl = moe.expert_range(rank, world, NE)
        keep = []
        lay = moe.Layer(d, F, NE, K, qt, L["router_w"], local_experts(moe, L, "gate", first, nl, keep),
                        local_experts(moe, L, "up", first, nl, keep),
                        local_experts(moe, L, "down", first, nl, keep),
                        first_expert=first, n_local=nl)

        def gather(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out

        moe.connect_expert_parallel(lay, rank, gather)
        moe.init_expert_parallel_comm(rank, world, gather)
        outs, inputs = [], []
        modes = sharded if isinstance(sharded, list) else [sharded] * len(token_counts)
        for T, shard in zip(token_counts, modes):
            if shard:
                x = orc.make_tokens(seed + T, world * T, d)[rank * T:(rank + 1) * T]
            else:
                x = orc.make_tokens(seed + T, T, d)
            inputs.append(x)
            dist.barrier()
            outs.append(lay.forward(x, flags=moe.EP_SHARDED if shard else 0))
        res = {"outs": outs}
        # this rank's own reference: one GPU with every expert, and the oracle
        if any(modes) or rank == 0:
            full = moe.Layer(d, F, NE, K, qt, L["router_w"], L["gate"], L["up"], L["down"])
            res["single"] = [full.forward(x) for x in inputs]
            res["oracle"] = [orc.moe_ffn(L, x)[0] for x in inputs]
            full.close()
        dist.barrier()   # no rank frees its exchange buffer while another may write to it
        lay.close()
        moe.shutdown()
        results[rank] = res
    except Exception as e:  # reported to the parent
        results[rank] = {"error": repr(e)}
    finally:
        dist.destroy_process_group()


def run_ranks(shape, token_counts, sharded):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_rank_main,
                       args=(world, free_port(), shape, token_counts, sharded, results),
                       nprocs=world, join=True, start_method="spawn")
    res = dict(results)
    for r in range(world):
        assert "error" not in res[r], res[r]
    return world, res


def assert_close(got, ref, T):
    err = float(np.abs(got - ref).max())
    rel = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
    assert err <= MAX_ABS and rel <= REL_L2, (T, err, rel)


SHAPES = [
    (2048, 1024, 16, 4, 1, 61),   # Q8_0, two-m-tile down items
    (2048, 2048, 8, 2, 2, 62),    # Q4_0, 2048-column down stages
]


@pytest.mark.parametrize("shape", SHAPES)
def test_expert_parallel_matches_one_gpu(shape):
    # repeated launches alternate exchange halves; 100 and 300 tokens take the
    # grouped GEMM and the NCCL all-reduce of the partial outputs
    token_counts = [1, 7, 32, 7, 100, 300, 5]
    world, res = run_ranks(shape, token_counts, sharded=False)
    for i, T in enumerate(token_counts):
        single = res[0]["single"][i]
        for r in range(world):
            np.testing.assert_array_equal(res[r]["outs"][i], res[0]["outs"][i])
            if T <= 64:   # the fused kernel's slot-order combine: bit-identical
                np.testing.assert_array_equal(res[r]["outs"][i], single)
            else:         # partial outputs summed across ranks: fp32 reassociation
                assert float(np.abs(res[r]["outs"][i] - single).max()) <= 1e-5
        assert_close(single, res[0]["oracle"][i], T)


@pytest.mark.parametrize("shape", SHAPES)
def test_token_sharded_matches_one_gpu(shape):
    # per-rank token counts: 1-32 run the fused kernel with the in-kernel
    # all-to-all; 100 and 300 the NCCL all-to-all around the grouped GEMMs
    token_counts = [1, 7, 32, 7, 100, 300, 5]
    world, res = run_ranks(shape, token_counts, sharded=True)
    for i, T in enumerate(token_counts):
        for r in range(world):
            got, single = res[r]["outs"][i], res[r]["single"][i]
            if T <= 64:   # the same per-pair arithmetic as one GPU's fused kernel
                np.testing.assert_array_equal(got, single)
            else:
                assert float(np.abs(got - single).max()) <= 1e-5, (T, r)
            assert_close(got, res[r]["oracle"][i], T)


def test_replicated_and_token_sharded_forwards_mixed_on_one_layer():
    """the two modes keep separate arrival counts: any order of them on one
    layer stays in step across the ranks"""
    shape = SHAPES[0]
    token_counts = [7, 5, 3, 32, 4, 100, 9, 2]
    modes = [False, True, False, True, True, True, False, True]
    world, res = run_ranks(shape, token_counts, sharded=modes)
    for i, (T, shard) in enumerate(zip(token_counts, modes)):
        for r in range(world):
            got = res[r]["outs"][i]
            if shard:
                single = res[r]["single"][i]
            else:
                np.testing.assert_array_equal(got, res[0]["outs"][i])
                single = res[0]["single"][i]
            if T <= 64:
                np.testing.assert_array_equal(got, single)
            else:
                assert float(np.abs(got - single).max()) <= 1e-5, (T, r)
            assert_close(got, res[r]["oracle"][i] if shard else res[0]["oracle"][i], T)
