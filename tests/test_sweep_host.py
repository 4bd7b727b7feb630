"""CPU tests of the layer sweep's multi-rank host logic with the gloo backend (world size 2):
deterministic LPT sharding, the metric all_gather, and failure detection when a rank dies before
the collective (the survivor gets an error within the process-group timeout instead of hanging)."""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tricast_b200.sweep import FORMATS, METRIC_FIELDS, SweepConfig, gather, results, shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_lpt_shard_covers_every_layer_once_and_balances():
    layers = SweepConfig().layers()
    assert len(layers) == 196
    for world in (1, 2, 4, 8):
        parts = [shard(layers, world, r) for r in range(world)]
        seen = sorted(e[0] for p in parts for e in p)
        assert seen == list(range(196))
        loads = [sum(e[2] * e[3] for e in p) for p in parts]
        assert max(loads) / min(loads) < 1.05
        assert parts == [shard(layers, world, r) for r in range(world)]  # deterministic


def _gather_worker(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    cfg = SweepConfig(blocks=2)
    layers = cfg.layers()
    mine = shard(layers, world, rank)
    sums = torch.zeros((len(mine), len(FORMATS), len(METRIC_FIELDS)), dtype=torch.float64)
    for row, e in enumerate(mine):
        sums[row, :, 0] = 1000.0 + e[0]          # signal
        sums[row, :, 2] = 1.0 + e[0] / 100.0    # error
        sums[row, :, 1] = 1000.0 + e[0]
        sums[row, :, 3] = 999.0 + e[0]
    table = gather(mine, sums, len(layers), world)
    if rank == 0:
        queue.put(table.tolist())
    dist.barrier()
    dist.destroy_process_group()


def test_gather_over_gloo_assembles_all_layers():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    table = torch.tensor(queue.get(timeout=120), dtype=torch.float64)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert table.shape == (14, len(FORMATS), len(METRIC_FIELDS))
    assert torch.equal(table[:, 0, 0], 1000.0 + torch.arange(14, dtype=torch.float64))
    recs = results(table, SweepConfig(blocks=2))
    assert recs[3]["mxfp4"]["sqnr_db"] > 0 and recs[3]["name"] == "model.layers.0.o_proj"


def _dying_worker(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # the rank dies between steps, before the metric gather
    cfg = SweepConfig(blocks=1)
    mine = shard(cfg.layers(), world, rank)
    sums = torch.zeros((len(mine), len(FORMATS), len(METRIC_FIELDS)), dtype=torch.float64)
    try:
        gather(mine, sums, len(cfg.layers()), world)
        queue.put("no error")
    except Exception as exc:  # noqa: BLE001 - the failure is what we test for
        queue.put(type(exc).__name__)


@pytest.mark.timeout(120)
def test_rank_failure_surfaces_as_error_not_hang():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_dying_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    outcome = queue.get(timeout=90)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert outcome != "no error"
    assert procs[1].exitcode == 3
