"""Failure detection of the expert-parallel exchange, without a GPU fault.

The fused decode kernel waits (bounded) for the other ranks' arrivals.  A
rank that is missing must turn into MOE_ERR_TIMEOUT from moe_layer_status,
with the device still usable afterwards:

* one GPU is enough for the first test: two processes share GPU 0, rank 1
  connects its exchange buffer and then never launches anything, so rank 0's
  kernel waits for arrivals that nothing sends; with the wait limit set to
  20 ms it must return MOE_ERR_TIMEOUT quickly (replicated and token-sharded
  forwards), and after moe_layer_ep_reset the same layer must still compute
  its experts' partial output correctly on the five-launch path.  Only one
  kernel ever waits, and it waits on a flag no kernel sets.
* with two or more GPUs, rank 1 skips one forward between steps (nothing of
  it in flight): rank 0 gets MOE_ERR_TIMEOUT, every rank resets between two
  host barriers, and the next forward is correct on every rank.
"""
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_package

pytestmark = pytest.mark.gpu

TIMEOUT = -7
SHAPE = (2048, 1024, 16, 4, 1, 71)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank, world, device):
    from oracle import oracle as orc
    moe = load_package()
    d, F, NE, K, qt, seed = SHAPE
    L = orc.make_layer(seed, d, F, NE, K, qt)
    moe.init(device)
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

    lay = moe.Layer(d, F, NE, K, qt, L["router_w"], local("gate"), local("up"), local("down"),
                    first_expert=first, n_local=nl)

    def gather(obj):
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    moe.connect_expert_parallel(lay, rank, gather)
    return orc, moe, L, lay, keep, (first, nl)


def _missing_peer(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        orc, moe, L, lay, keep, (first, nl) = _setup(rank, world, 0)
        res = {}
        if rank == 0:
            lay.set_wait_ms(20)
            x = orc.make_tokens(5, 4, SHAPE[0])
            for name, flags in (("replicated", 0), ("sharded", moe.EP_SHARDED)):
                t0 = time.perf_counter()
                try:
                    lay.forward(x, flags=flags)
                    res[name] = ("no error", 0.0)
                except moe.MoeError as e:
                    res[name] = (e.code, time.perf_counter() - t0)
                lay.ep_reset()
            # the layer and the device still work: the five-launch path gives
            # this rank's experts' share of the output (no peer involved)
            part = lay.forward(x, flags=moe.NO_FUSE)
            z, _, _ = orc.moe_slot_terms(L, x, first, nl)
            ref = orc.combine_slot_terms(z, x.shape[0], SHAPE[3])
            res["partial_err"] = float(np.abs(part - ref).max())
            res["status_after"] = lay.status()
        dist.barrier()   # rank 1 keeps its buffer mapped until rank 0 is done
        lay.close()
        results[rank] = res
    except Exception as e:
        results[rank] = {"error": repr(e)}
    finally:
        dist.destroy_process_group()


def test_missing_rank_times_out_and_device_recovers():
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_missing_peer, args=(2, free_port(), results), nprocs=2, join=True,
                       start_method="spawn")
    res = dict(results)
    for r in range(2):
        assert "error" not in res[r], res[r]
    for name in ("replicated", "sharded"):
        code, secs = res[0][name]
        assert code == TIMEOUT, (name, code)
        assert secs < 5.0, (name, secs)
    assert res[0]["partial_err"] <= 2e-3
    assert res[0]["status_after"] == 0


def _skipped_step(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        orc, moe, L, lay, keep, _ = _setup(rank, world, rank)
        lay.set_wait_ms(300)
        x = orc.make_tokens(9, 8, SHAPE[0])
        ref = orc.moe_ffn(L, x)[0]
        codes = []
        for step in range(3):
            dist.barrier()
            if step == 1 and rank == 1:
                codes.append("skipped")
            else:
                try:
                    out = lay.forward(x)
                    codes.append(float(np.abs(out - ref).max()))
                except moe.MoeError as e:
                    codes.append(e.code)
            if step == 1:
                # recovery: every rank resets between two host barriers
                dist.barrier()
                lay.ep_reset()
                dist.barrier()
        dist.barrier()
        lay.close()
        results[rank] = {"codes": codes}
    except Exception as e:
        results[rank] = {"error": repr(e)}
    finally:
        dist.destroy_process_group()


def test_skipped_forward_times_out_then_ranks_recover():
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two or more GPUs")
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_skipped_step, args=(world, free_port(), results), nprocs=world,
                       join=True, start_method="spawn")
    res = dict(results)
    for r in range(world):
        assert "error" not in res[r], res[r]
    assert res[0]["codes"][1] == TIMEOUT
    for r in range(world):
        codes = res[r]["codes"]
        assert isinstance(codes[0], float) and codes[0] <= 2e-3, (r, codes)
        assert isinstance(codes[2], float) and codes[2] <= 2e-3, (r, codes)
