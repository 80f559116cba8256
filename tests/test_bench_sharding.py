"""Host logic of bench.py's multi-GPU runs, on the CPU: the contiguous per-rank sequence
slices of the strong-scaling run cover every named shape exactly once, and the timing
all-reduce (max over ranks) agrees on two gloo ranks (the NCCL runs use the same calls)."""
from __future__ import annotations

import importlib.util
import os
import socket
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("semx_bench_shard", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("S", [404, 1284, 1, 7, 0])
@pytest.mark.parametrize("W", [1, 2, 4, 8])
def test_shards_partition_the_sequences(S, W):
    bench = _bench()
    sizes = [bench._shard(S, r, W) for r in range(W)]
    assert sum(sizes) == S
    assert all(z >= 0 for z in sizes) and max(sizes) - min(sizes) <= 1
    starts = [r * S // W for r in range(W)]
    assert starts == [sum(sizes[:r]) for r in range(W)]  # contiguous, in rank order


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        bench = _bench()
        ms = bench._max_over_ranks(10.0 + rank, world, torch.device("cpu"))
        S = 404
        lo = rank * S // world
        hi = lo + bench._shard(S, rank, world)
        got = torch.tensor([lo, hi], dtype=torch.int64)
        allv = [torch.zeros(2, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(allv, got)
        out[rank] = (ms, [tuple(v.tolist()) for v in allv])
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_agree_on_timing_and_slices():
    world = 2
    port = _free_port()
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_rank_main, args=(world, port, out), nprocs=world, start_method="spawn", join=True)
    assert out[0][0] == out[1][0] == 11.0
    assert out[0][1] == out[1][1] == [(0, 202), (202, 404)]
