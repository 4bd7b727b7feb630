"""CPU tests of the N-column split's host logic: the slab partition, the all-reduce of the shards'
amax bits (gloo, world size 2) and the all-gather that assembles the full output."""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tricast_b200.shard import column_slab, gather_columns, needs_tensor_amax, reduce_amax_bits
from tricast_b200.spec import SCHEMES


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n", [1, 7, 512, 4096, 4097, 12288])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_column_slabs_tile_the_columns(n, world):
    slabs = [column_slab(n, world, r) for r in range(world)]
    assert slabs[0][0] == 0 and slabs[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(slabs, slabs[1:]))
    widths = [e - s for s, e in slabs]
    assert max(widths) - min(widths) <= 1


def test_column_slab_rejects_bad_ranks():
    with pytest.raises(ValueError):
        column_slab(16, 2, 2)


def test_which_schemes_need_the_tensor_amax():
    assert needs_tensor_amax(SCHEMES["nvfp4"]) and needs_tensor_amax(SCHEMES["fp8_tensor"])
    assert not needs_tensor_amax(SCHEMES["mxfp4"]) and not needs_tensor_amax(SCHEMES["int4_g128_zp"])
    assert not needs_tensor_amax(SCHEMES["int8_row"])


def _amax_bits(x: np.ndarray) -> int:
    """NaN-propagating amax as fp32 bits (what tc_tensor_amax_bits computes)."""
    return int((x.astype(np.float32).view(np.uint32) & 0x7FFFFFFF).max())


def _worker(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    rng = np.random.default_rng(rank)
    shard = rng.standard_normal((8, 16)).astype(np.float32) * (3.0 if rank == 1 else 1.0)
    bits = torch.tensor(_amax_bits(shard), dtype=torch.int32)
    got = float(reduce_amax_bits(bits).view(torch.float32))
    nan_bits = torch.tensor(_amax_bits(np.array([np.nan if rank == 0 else 1.0], np.float32)), dtype=torch.int32)
    got_nan = float(reduce_amax_bits(nan_bits).view(torch.float32))
    m, n = 5, 11
    full = torch.arange(m * n, dtype=torch.float32).reshape(m, n)
    s, e = column_slab(n, world, rank)
    gathered = gather_columns(full[:, s:e].contiguous(), n)
    queue.put((rank, got, float(np.abs(shard).max()), got_nan, bool(torch.equal(gathered, full))))
    dist.barrier()
    dist.destroy_process_group()


def test_amax_reduce_and_column_gather_over_gloo():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    global_amax = max(r[2] for r in results)
    for _, got, _, got_nan, gathered_ok in results:
        assert got == global_amax       # every rank holds the global amax
        assert np.isnan(got_nan)        # NaN propagates through the integer max
        assert gathered_ok
