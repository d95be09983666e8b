"""The multi-GPU group's host logic without a GPU: the frame split
(tpmd_shard_range) and the NCCL communicator set-up with its failure
handling (non-blocking init polled under a wall-clock limit, abort on expiry
or on an asynchronous error), run against a fake NCCL inside libtpmd.so."""
from __future__ import annotations

import pytest

import tpmd
from tpmd import multi


@pytest.mark.parametrize("n,world", [(750, 8), (750, 3), (50, 4), (5, 8), (1, 2), (0, 4), (96, 1)])
def test_shard_range_matches_python_split(n, world):
    got = [tpmd.shard_range(n, world, r) for r in range(world)]
    assert got == [multi.frame_range(n, world, r) for r in range(world)]
    assert sum(hi - lo for lo, hi in got) == n
    if world > 1 and n >= world:
        assert max(hi - lo for lo, hi in got) == -(-n // world)


def test_shard_range_rejects_bad_arguments():
    for args in ((-1, 2, 0), (10, 0, 0), (10, 2, 2), (10, 2, -1)):
        with pytest.raises(ValueError):
            tpmd.shard_range(*args)


def test_nccl_init_succeeds_after_polling():
    rc, aborts, msg = tpmd.nccl_selftest(4, 0, 5.0)
    assert rc == 0 and aborts == 0, msg


def test_nccl_init_times_out_and_aborts():
    rc, aborts, msg = tpmd.nccl_selftest(4, 1, 0.2)
    assert rc == -1
    assert "timed out" in msg
    assert aborts == 4


def test_nccl_async_error_aborts_every_communicator():
    rc, aborts, msg = tpmd.nccl_selftest(3, 2, 5.0)
    assert rc == -1
    assert "fake NCCL error" in msg
    assert aborts == 3


def test_nccl_init_call_failure_aborts_what_was_made():
    rc, aborts, msg = tpmd.nccl_selftest(3, 3, 5.0)
    assert rc == -1
    assert "ncclCommInitRankConfig" in msg
    assert aborts == 1  # rank 0 had been created before rank 1's call failed
