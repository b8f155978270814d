"""Host side of the head-sharded step on CPU ranks (gloo, world size 2).

A model whose KV heads are sharded over ranks runs the single-GPU step on
each rank's heads; the only exchange is the lazy decision of backend.py:446
(`accept_mask.all()` over every head), all-reduced with MIN between the
selection and the attention halves of the step. These tests run that
exchange on real gloo process groups: the head partition, the reduction for
every combination of local decisions, and a rank that fails before the
exchange (the survivor must get an error from its collective within the
group's timeout, not hang). No GPU is involved.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cvsa.backend import exchange_decision, shard_heads


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _exchange_worker(rank, world, port, local, results):
    _init(rank, world, port, 30)
    try:
        word = torch.tensor([local[rank]], dtype=torch.int32)
        exchange_decision(word, None)
        results[rank] = int(word.item())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("local", [(1, 1), (1, 0), (0, 1), (0, 0)])
def test_decision_exchange_is_min_over_ranks(local):
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_exchange_worker, args=(2, _free_port(), local, results), nprocs=2,
                       join=True, start_method="spawn")
    want = min(local)
    assert dict(results) == {0: want, 1: want}


def _fault_worker(rank, world, port, results):
    _init(rank, world, port, 3)
    if rank == 1:
        # this rank fails between steps, before the exchange, and never joins it
        results[1] = "left"
        return
    word = torch.tensor([1], dtype=torch.int32)
    try:
        exchange_decision(word, None)
        results[0] = "completed"
    except Exception as e:  # noqa: BLE001 - any collective error is the expected outcome
        results[0] = "error: " + type(e).__name__


def test_rank_lost_before_exchange_surfaces_as_error():
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    procs = mp.start_processes(_fault_worker, args=(2, _free_port(), results), nprocs=2,
                               join=False, start_method="spawn")
    for p in procs.processes:
        p.join(120)
    assert all(not p.is_alive() for p in procs.processes), "a rank hung"
    assert results.get(1) == "left"
    assert str(results.get(0, "")).startswith("error"), results.get(0)


def test_shard_heads_partition():
    kv, qs = zip(*(shard_heads(8, 64, r, 8) for r in range(8)))
    assert [s.start for s in kv] == list(range(8)) and all(s.stop - s.start == 1 for s in kv)
    assert [(s.start, s.stop) for s in qs] == [(8 * r, 8 * r + 8) for r in range(8)]
    kv2, q2 = shard_heads(8, 32, 1, 2)
    assert (kv2.start, kv2.stop, q2.start, q2.stop) == (4, 8, 16, 32)
    with pytest.raises(ValueError):
        shard_heads(8, 32, 0, 3)
