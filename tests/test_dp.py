"""Data-parallel partitioning and the host group (CPU only; the multi-rank test runs two gloo ranks)."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from belt_b200 import dp, synth


def test_lpt_covers_every_request_once_with_equal_counts():
    lens = synth.log_uniform_lengths(1024, 1024, 65536)
    for world in (1, 2, 3, 4, 8):
        parts = dp.partition_lpt(lens, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(len(lens)))
        counts = [len(p) for p in parts]
        assert max(counts) - min(counts) <= 1


def test_lpt_balances_tokens_better_than_even_split():
    lens = synth.log_uniform_lengths(1024, 1024, 65536)
    for world in (2, 4, 8):
        lpt = dp.imbalance(lens, dp.partition_lpt(lens, world))
        even = dp.imbalance(lens, dp.partition_even(lens, world))
        assert lpt <= even
        assert lpt < 1.01, lpt                     # 128+ requests per rank: within 1 % of the mean


def test_lpt_edge_cases():
    assert dp.partition_lpt([], 4) == [[], [], [], []]
    assert dp.partition_lpt([5], 3) == [[0], [], []]
    assert dp.partition_lpt([7, 7, 7, 7], 2) == [[0, 2], [1, 3]]    # deterministic ties
    with pytest.raises(ValueError):
        dp.partition_lpt([1, 2], 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, lens, out):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    g = dp.HostGroup(timeout_s=60)
    mine = dp.partition_lpt(lens, world)[g.rank]
    tokens = sum(lens[i] for i in mine)
    g.barrier()
    out[rank] = (mine, g.max(float(rank * 10 + 1)), g.sum(float(tokens)))
    g.close()


def test_host_group_two_gloo_ranks():
    """Two ranks agree on the partition without exchanging it, and max / sum over ranks are right."""
    lens = synth.log_uniform_lengths(256, 1024, 65536)
    world, port = 2, _free_port()
    out = mp.Manager().dict()
    mp.spawn(_rank_main, args=(world, port, lens, out), nprocs=world, join=True)
    shares = [out[r][0] for r in range(world)]
    assert sorted(i for s in shares for i in s) == list(range(len(lens)))
    assert all(out[r][1] == 11.0 for r in range(world))
    assert all(out[r][2] == float(sum(lens)) for r in range(world))


def test_host_group_single_rank_is_local():
    g = dp.HostGroup()
    assert g.world == 1 and g.dist is None and g.max(3.5) == 3.5 and g.sum(2.0) == 2.0
    g.barrier()
    g.close()


def _lonely_rank(rank, world, port, out):
    if rank == 1:
        return                                    # this rank never joins
    os.environ.update(RANK="0", WORLD_SIZE=str(world), LOCAL_RANK="0", MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    try:
        dp.HostGroup(timeout_s=3)
        out[0] = "joined"
    except Exception as e:                        # the launcher's store gives up: an error, not a hang
        out[0] = type(e).__name__


def test_host_group_missing_rank_fails_instead_of_hanging():
    out = mp.Manager().dict()
    mp.spawn(_lonely_rank, args=(2, _free_port(), out), nprocs=2, join=True)
    assert out[0] != "joined"
