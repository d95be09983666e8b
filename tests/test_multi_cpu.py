"""Host logic of the multi-GPU path on gloo ranks (CPU): frame sharding
covers a clip exactly once, arena bytes broadcast from rank 0, max-over-ranks
timing, the pipelined end-to-end schedule (every frame decoded once, by the
planned rank, from the styles of its own chunk, with the same collective
steps on every rank), and a rank that fails before the broadcast is seen by
the other through a short process-group timeout rather than a hang."""
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


def test_pipeline_plan_covers_each_chunk_once():
    for n in (0, 1, 49, 50, 51, 750, 751):
        for world in (1, 2, 3, 4, 8):
            plan = multi.pipeline_plan(n, world)
            assert len(plan) == -(-n // 50)
            for k, ranges in enumerate(plan):
                assert len(ranges) == world
                got = sorted(r for r in ranges if r[1] > r[0])
                f0, f1 = 50 * k, min(n, 50 * k + 50)
                assert got[0][0] == f0 and got[-1][1] == f1
                assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
                if world >= 3:
                    assert ranges[0][1] == ranges[0][0]  # rank 0 only samples
                    sizes = [hi - lo for lo, hi in ranges[1:]]
                    assert max(sizes) - min(sizes) <= 1
            total = sum(multi.frames_per_rank(plan, r) for r in range(world))
            assert total == n
    p2 = multi.pipeline_plan(750, 2)
    assert multi.frames_per_rank(p2, 0) == 100 and multi.frames_per_rank(p2, 1) == 650
    assert [multi.frames_per_rank(multi.pipeline_plan(750, 8), r) for r in range(8)] == [0, 108] + [107] * 6
    with pytest.raises(ValueError):
        multi.pipeline_plan(10, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init_gloo(rank, world, port, collective_s):
    """gloo process group whose rendezvous waits up to 120 s for ranks that
    start late (spawned processes importing torch on a loaded host), while
    its collectives time out after collective_s"""
    import datetime
    import torch.distributed as dist
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=120))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=collective_s))


def _worker(rank, world, port, mode, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        _init_gloo(rank, world, port, 10)
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


class _FakeDecoder:
    """decode_ptr writes each frame's style[0] into the first float of the
    frame; the feats arena is a small byte tensor."""

    def __init__(self, rank):
        self.feats = torch.arange(64, dtype=torch.uint8) if rank == 0 else torch.zeros(64, dtype=torch.uint8)
        self.adopted = False

    def adopt_arena(self, which):
        self.adopted = which == 1

    def decode_ptr(self, sp, n, op):
        import ctypes
        import numpy as np
        st = np.ctypeslib.as_array((ctypes.c_float * (n * 512)).from_address(sp)).reshape(n, 512)
        for i in range(n):
            ctypes.c_float.from_address(op + i * multi.FRAME_BYTES).value = float(st[i, 0])


class _FakePipeline:
    """styles_cb over `n` frames in chunks of `chunk`: style of frame t is t."""

    def __init__(self, n, chunk):
        self.n, self.chunk = n, chunk

    def styles_cb(self, image, audio, emotion, cb, noise=None, seed=0):
        import numpy as np
        for f0 in range(0, self.n, self.chunk):
            f1 = min(self.n, f0 + self.chunk)
            st = np.repeat(np.arange(f0, f1, dtype=np.float32)[:, None], 512, axis=1)
            if cb(f0, st):
                break
        return self.n


def _pipe_worker(rank, world, port, n, chunk, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        _init_gloo(rank, world, port, 30)
        multi.arena_tensor = lambda dec, which, device: dec.feats
        multi.FRAME_BYTES = 16  # a 4-float frame keeps the buffers small
        dec = _FakeDecoder(rank)
        plan = multi.pipeline_plan(n, world, chunk)
        m = max(multi.frames_per_rank(plan, rank), 1)
        frames = torch.zeros((m, 4))
        got = multi.generate_pipelined(rank, world, "cpu", n, dec, frames,
                                       pipe=_FakePipeline(n, chunk) if rank == 0 else None, chunk=chunk)
        marks = [float(frames[i, 0]) for i in range(got)]
        feats_ok = bool(torch.equal(dec.feats, torch.arange(64, dtype=torch.uint8))) and (rank == 0 or dec.adopted)
        q.put((rank, "ok", marks, feats_ok))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, "error", type(e).__name__ + ": " + str(e)[:300], None))


@pytest.mark.parametrize("world,n", [(1, 23), (2, 71), (3, 23), (4, 95)])
def test_pipelined_generation_gloo(world, n):
    chunk = 10
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pipe_worker, args=(r, world, port, n, chunk, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert all(o[1] == "ok" for o in out), out
    plan = multi.pipeline_plan(n, world, chunk)
    for rank, _, marks, feats_ok in out:
        want = [float(t) for ranges in plan for lo, hi in (ranges[rank],) for t in range(lo, hi)]
        assert marks == want, (rank, marks, want)
        assert feats_ok
    assert sorted(m for o in out for m in o[2]) == [float(t) for t in range(n)]


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
