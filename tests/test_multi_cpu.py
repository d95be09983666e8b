"""Host logic of the multi-GPU path on 2 gloo ranks (CPU): frame sharding
covers a clip exactly once, arena bytes broadcast from rank 0, max-over-ranks
timing, and a rank that fails before the broadcast is seen by the other
through a short process-group timeout rather than a hang."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from tpmd import multi


def test_frame_ranges_cover_clip():
    for n in (0, 1, 49, 50, 750, 751):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                a, b = multi.frame_range(n, world, r)
                assert 0 <= a <= b <= n
                for s, e in multi.sub_batches(a, b, 50):
                    assert 0 < e - s <= 50
                    seen.extend(range(s, e))
            assert seen == list(range(n)), (n, world)
    assert multi.frame_range(750, 8, 7) == (658, 750)
    with pytest.raises(ValueError):
        multi.frame_range(10, 2, 2)
    with pytest.raises(ValueError):
        multi.sub_batches(0, 10, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=10))
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure on rank 1 before the broadcast")
        arena = torch.arange(4096, dtype=torch.uint8) if rank == 0 else torch.zeros(4096, dtype=torch.uint8)
        multi.broadcast_bytes(arena, src=0)
        ok = bool(torch.equal(arena, torch.arange(4096, dtype=torch.uint8)))
        worst = multi.max_over_ranks(10.0 + rank)
        a, b = multi.frame_range(750, world, rank)
        q.put((rank, "ok", ok, worst, (a, b)))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, never hangs it
        q.put((rank, "error", type(e).__name__, str(e)[:200], None))


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(out)


def test_broadcast_and_max_over_ranks_gloo():
    out = _run("ok")
    assert [o[1] for o in out] == ["ok", "ok"], out
    assert all(o[2] for o in out)
    assert all(o[3] == 11.0 for o in out)
    assert out[0][4] == (0, 375) and out[1][4] == (375, 750)


def test_failed_rank_is_reported_not_hung():
    out = _run("fail")
    assert out[1][1] == "error" and "injected" in out[1][3]
    # rank 0's broadcast ends with an error (peer gone / timeout), not a hang
    assert out[0][1] == "error", out
