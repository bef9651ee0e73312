"""Expert parallelism on the CPU: the decompositions the GPU path uses across
GPUs, run by gloo ranks with the oracle.

Each rank computes the combine terms y / (1 / w) of the (token, slot) pairs
whose expert it owns (expert_range), the ranks exchange their rows (here an
all-gather, on the GPUs direct NVLink stores), and every rank adds each
token's rows in slot order.  The result must equal the single-process
oracle bit for bit on every rank.  Batches above 64 tokens instead sum
the ranks' partial outputs (an all-reduce): identical on every rank and
within fp32 reassociation of the oracle.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_package


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, case, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as orc
        moe = load_package()
        d, F, NE, K, qt, T, seed, renorm = case
        L = orc.make_layer(seed, d, F, NE, K, qt, renorm=renorm, zipf=not renorm)
        x = orc.make_tokens(seed, T, d)
        first, nl = moe.expert_range(rank, world, NE)
        z, ids, w = orc.moe_slot_terms(L, x, first, nl)
        # rows of experts owned elsewhere are zero here; exactly one rank owns each row
        rows = torch.from_numpy(z)
        gathered = [torch.empty_like(rows) for _ in range(world)]
        dist.all_gather(gathered, rows)
        owner = np.array([[moe.expert_range(r, world, NE)[0] <= e < sum(moe.expert_range(r, world, NE))
                           for r in range(world)] for e in ids.reshape(-1)])
        assert (owner.sum(axis=1) == 1).all()
        full = np.stack([g.numpy() for g in gathered])[owner.argmax(axis=1), np.arange(T * K)]
        out = orc.combine_slot_terms(full, T, K)
        ref, *_ = orc.moe_ffn(L, x)
        results[rank] = bool(np.array_equal(out, ref))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("case", [
    (256, 128, 16, 4, 1, 9, 4, False),   # Q8_0, Zipf-skewed router
    (512, 256, 8, 2, 2, 5, 3, True),     # Q4_0, Mixtral-style renormalised top-2
])
def test_expert_parallel_decomposition_is_exact(world, case):
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_rank_main, args=(world, free_port(), case, results), nprocs=world,
                       join=True, start_method="spawn")
    assert dict(results) == {r: True for r in range(world)}


def _rank_partial(rank, world, port, case, results):
    """larger batches: each rank's partial output (slot-order combine of its
    own experts' rows), summed across the ranks as the NCCL all-reduce does"""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as orc
        moe = load_package()
        d, F, NE, K, qt, T, seed, renorm = case
        L = orc.make_layer(seed, d, F, NE, K, qt, renorm=renorm, zipf=not renorm)
        x = orc.make_tokens(seed, T, d)
        first, nl = moe.expert_range(rank, world, NE)
        z, ids, w = orc.moe_slot_terms(L, x, first, nl)
        part = torch.from_numpy(orc.combine_slot_terms(z, T, K))
        dist.all_reduce(part)
        ref, *_ = orc.moe_ffn(L, x)
        results[rank] = (part.numpy().tobytes(), float(np.abs(part.numpy() - ref).max()),
                         float(np.abs(ref).max()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_partial_sums_match_oracle(world):
    case = (256, 128, 16, 4, 1, 70, 5, False)
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_rank_partial, args=(world, free_port(), case, results), nprocs=world,
                       join=True, start_method="spawn")
    res = dict(results)
    assert len({res[r][0] for r in range(world)}) == 1      # identical on every rank
    err, scale = res[0][1], res[0][2]
    assert err <= 1e-6 * max(scale, 1.0)                     # fp32 reassociation only


def _rank_sharded(rank, world, port, case, results):
    """token-sharded: rank r holds rows [r*T, (r+1)*T) of one global batch.
    The ranks gather every rank's tokens (on the GPUs: tokens and ids written
    into every rank's exchange buffer), each computes the combine terms of
    the pairs of ALL tokens whose expert it owns, the rows go back to the
    ranks that own the tokens (on the GPUs: stored straight into the owner's
    buffer; here an all-to-all), and each rank combines its own tokens in
    slot order.  Must equal the oracle on the global batch bit for bit."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as orc
        moe = load_package()
        d, F, NE, K, qt, T, seed, renorm = case
        L = orc.make_layer(seed, d, F, NE, K, qt, renorm=renorm, zipf=not renorm)
        x_all = orc.make_tokens(seed, world * T, d)
        mine = torch.from_numpy(np.ascontiguousarray(x_all[rank * T:(rank + 1) * T]))
        got = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(got, mine)                       # dispatch: every rank's tokens
        xg = torch.cat(got).numpy()
        first, nl = moe.expert_range(rank, world, NE)
        z, ids, w = orc.moe_slot_terms(L, xg, first, nl)  # rows of the local experts
        z = torch.from_numpy(z.reshape(world, T * K, d).copy())
        back = [torch.empty_like(z[0]) for _ in range(world)]
        for q in range(world):                           # combine: rows to their tokens' ranks
            dist.scatter(back[q], list(z.unbind(0)) if q == rank else None, src=q)
        # rows of my tokens from every rank: exactly one rank owns each row
        own_ids = ids.reshape(world, T * K)[rank]
        owner = np.array([[moe.expert_range(r, world, NE)[0] <= e <
                           sum(moe.expert_range(r, world, NE)) for r in range(world)]
                          for e in own_ids])
        assert (owner.sum(axis=1) == 1).all()
        rows = torch.stack(back).numpy()[owner.argmax(axis=1), np.arange(T * K)]
        out = orc.combine_slot_terms(rows, T, K)
        ref, *_ = orc.moe_ffn(L, x_all)
        results[rank] = bool(np.array_equal(out, ref[rank * T:(rank + 1) * T]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("case", [
    (256, 128, 16, 4, 1, 6, 8, False),   # Q8_0, Zipf-skewed router
    (512, 256, 8, 2, 2, 4, 9, True),     # Q4_0, Mixtral-style renormalised top-2
])
def test_token_sharded_decomposition_is_exact(world, case):
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_rank_sharded, args=(world, free_port(), case, results), nprocs=world,
                       join=True, start_method="spawn")
    assert dict(results) == {r: True for r in range(world)}


@pytest.mark.parametrize("world,ne", [(2, 64), (3, 64), (8, 64), (8, 8), (7, 16)])
def test_expert_range_covers_every_expert_once(world, ne):
    moe = load_package()
    seen = []
    for r in range(world):
        first, nl = moe.expert_range(r, world, ne)
        assert nl >= ne // world
        seen += list(range(first, first + nl))
    assert seen == list(range(ne))
