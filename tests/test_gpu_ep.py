"""Expert parallelism on 2+ GPUs: every rank owns a contiguous range of
experts.  Decode batches run the fused decode kernel, which writes the rows
of its experts into the other ranks' exchange buffers over NVLink; larger
batches run the grouped GEMMs on the local experts and sum the ranks'
partial outputs with the library's NCCL all-reduce.  Every rank's output
must be the full layer output: identical across ranks, identical to one GPU
(decode) or within fp32 reassociation of it (larger batches), and within the
tolerance of the CPU oracle.

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


def _rank_main(rank, world, port, shape, token_counts, results):
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

        def local(name):
            ptrs = []
            for e in range(NE):
                if first <= e < first + nl:
                    b = moe.DeviceBuffer.from_numpy(np.ascontiguousarray(L[name][e]))
                    keep.append(b)
                    ptrs.append(b.ptr)
                else:
                    ptrs.append(0)
            return ptrs

        lay = moe.Layer(d, F, NE, K, qt, L["router_w"], local("gate"), local("up"),
                        local("down"), first_expert=first, n_local=nl)

        def gather(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out

        moe.connect_expert_parallel(lay, rank, gather)
        moe.init_expert_parallel_comm(rank, world, gather)
        outs = []
        for T in token_counts:
            x = orc.make_tokens(seed + T, T, d)
            outs.append(lay.forward(x))
        res = {"outs": outs}
        if rank == 0:
            full = moe.Layer(d, F, NE, K, qt, L["router_w"], L["gate"], L["up"], L["down"])
            res["single"] = [full.forward(orc.make_tokens(seed + T, T, d)) for T in token_counts]
            res["oracle"] = [orc.moe_ffn(L, orc.make_tokens(seed + T, T, d))[0]
                             for T in token_counts]
            full.close()
        dist.barrier()   # no rank frees its exchange buffer while another may write to it
        lay.close()
        results[rank] = res
    except Exception as e:  # reported to the parent
        results[rank] = {"error": repr(e)}
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shape", [
    (2048, 1024, 16, 4, 1, 61),   # Q8_0, two-m-tile down items
    (2048, 2048, 8, 2, 2, 62),    # Q4_0, 2048-column down stages
])
def test_expert_parallel_matches_one_gpu(shape):
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    # repeated launches alternate exchange halves; 100 and 300 tokens take the
    # grouped GEMM and the NCCL all-reduce of the partial outputs
    token_counts = [1, 7, 32, 7, 100, 300, 5]
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_rank_main, args=(world, free_port(), shape, token_counts, results),
                       nprocs=world, join=True, start_method="spawn")
    res = dict(results)
    for r in range(world):
        assert "error" not in res[r], res[r]
    for i, T in enumerate(token_counts):
        single = res[0]["single"][i]
        ref = res[0]["oracle"][i]
        for r in range(world):
            np.testing.assert_array_equal(res[r]["outs"][i], res[0]["outs"][i])
            if T <= 64:   # the fused kernel's slot-order combine: bit-identical
                np.testing.assert_array_equal(res[r]["outs"][i], single)
            else:         # partial outputs summed across ranks: fp32 reassociation
                assert float(np.abs(res[r]["outs"][i] - single).max()) <= 1e-5
        err = float(np.abs(single - ref).max())
        rel = float(np.linalg.norm(single - ref) / np.linalg.norm(ref))
        assert err <= MAX_ABS and rel <= REL_L2, (T, err, rel)
