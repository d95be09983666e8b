"""The host decode's split schedule (tpmd_decode_schedule, host code only):
the groups cover the frames in order, never straddle a max_batch chunk (the
workspace holds one chunk), every group's parts cover it, and the config-2
call (50 frames, max_batch 50) gets the schedule measured on the B200: f32
frames in two groups (38 frames in parts 8, 10, 10, 10; 12 frames in parts
of 3), RGB24 frames in one group (29, 7, 7, 7)."""
from __future__ import annotations

import pytest

import tpmd


@pytest.mark.parametrize("rgb", [False, True])
@pytest.mark.parametrize("max_batch", [1, 2, 7, 8, 16, 24, 50, 64])
def test_groups_cover_frames_within_chunks(max_batch, rgb):
    for n in range(4, 181):
        plan = tpmd.decode_schedule(n, max_batch, rgb)
        f = 0
        for f0, g, parts in plan:
            assert f0 == f, (n, max_batch, plan)
            assert 1 <= g <= max_batch
            assert f0 // max_batch == (f0 + g - 1) // max_batch, "group straddles a chunk"
            assert parts and min(parts) >= 1 and sum(parts) == g
            f += g
        assert f == n


@pytest.mark.parametrize("max_batch", [16, 24, 50, 64])
def test_last_chunk_of_f32_frames_ends_in_short_parts(max_batch):
    """with 16 or more frames in the last chunk, its second group holds about
    a quarter of them in parts of two to four frames"""
    for n in range(16, 3 * max_batch + 1):
        m = n - ((n - 1) // max_batch) * max_batch  # frames in the last chunk
        if m < 16:
            continue
        plan = tpmd.decode_schedule(n, max_batch, False)
        f0, g, parts = plan[-1]
        assert g == max(2, round(0.24 * m) if (0.24 * m) % 1 != 0.5 else int(0.24 * m + 0.5)), (n, m, plan)
        assert all(2 <= p <= 4 for p in parts), (n, plan)
        assert plan[-2][0] + plan[-2][1] == f0


def test_config2_schedules():
    assert tpmd.decode_schedule(50, 50, False) == [(0, 38, [8, 10, 10, 10]), (38, 12, [3, 3, 3, 3])]
    assert tpmd.decode_schedule(50, 50, True) == [(0, 50, [29, 7, 7, 7])]
    # beyond one chunk: whole chunks first, each starting with a short part
    plan = tpmd.decode_schedule(120, 50, False)
    assert [(f0, g) for f0, g, _ in plan] == [(0, 50), (50, 50), (100, 15), (115, 5)]
    assert plan[0][2] == [11, 13, 13, 13]


def test_rejects_what_has_no_split_schedule():
    for n, mb in ((3, 50), (1, 8), (10, 0)):
        with pytest.raises(ValueError):
            tpmd.decode_schedule(n, mb)
    L = tpmd.load_library()
    import ctypes as C
    buf = (C.c_int64 * 4)()
    assert L.tpmd_decode_schedule(50, 50, 0, buf, 4) == -1  # too small a buffer
