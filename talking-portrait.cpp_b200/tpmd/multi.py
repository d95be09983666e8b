"""Frame sharding across GPUs (one process per GPU, torch.distributed).

Every frame is independent given the shared decoder weights and the
portrait's feature pyramid, so the decoder shards by frame with no
data-path collective:

* rank 0 prepares the weight arena and uploads the feats; both arenas are
  broadcast once, as raw bytes, over the process group (NCCL over
  NVLink/NVSwitch on a GPU box) and adopted by the other ranks;
* a clip of n frames is split into contiguous per-rank ranges of
  ceil(n / world) frames (the last rank takes the remainder), decoded in
  sub-batches of at most `batch` frames, written straight into each rank's
  slice of the caller's frame buffer;
* device time is reduced as the max over ranks.

End to end (generate_pipelined) the serial stages (encoders, sampler) run on
rank 0 and the decode overlaps them: the sampler hands over each chunk's
styles as soon as they exist (tppl_styles_cb), rank 0 broadcasts them, and
the other ranks decode their share of the chunk while the next one is
sampled.

The reference has no multi-GPU path (src/pipeline.cpp:153-184 decodes
batches serially on one device, after sampling every chunk); this module is
new.
"""
from __future__ import annotations


def frame_range(n_frames: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of the frames `rank` decodes: contiguous blocks of
    ceil(n / world); trailing ranks may get fewer (or none)."""
    if n_frames < 0 or world < 1 or not 0 <= rank < world:
        raise ValueError("bad shard arguments")
    per = -(-n_frames // world)
    start = min(n_frames, rank * per)
    return start, min(n_frames, start + per)


def sub_batches(start: int, stop: int, batch: int) -> list[tuple[int, int]]:
    """[start, stop) split into dispatches of at most `batch` frames."""
    if batch < 1:
        raise ValueError("batch must be >= 1")
    return [(s, min(stop, s + batch)) for s in range(start, stop, batch)]


class _DeviceBytes:
    """__cuda_array_interface__ view of a device byte range (no copy)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3}


def arena_tensor(dec, which: int, device):
    """A torch uint8 CUDA tensor aliasing one of the decoder's arenas
    (0: prepared weights, 1: feats)."""
    import torch
    ptr, n = dec.arena(which)
    return torch.as_tensor(_DeviceBytes(ptr, n), device=device)


def broadcast_bytes(t, src: int = 0, group=None) -> None:
    """Broadcast a byte tensor from `src` (in place on every rank)."""
    import torch.distributed as dist
    dist.broadcast(t, src=src, group=group)


def share_decoder(dec, rank: int, device, group=None) -> None:
    """Make every rank's decoder ready from rank 0's prepared arenas: rank 0
    must have run prepare() and set_feats(); the others adopt the bytes."""
    import torch
    for which in (0, 1):
        t = arena_tensor(dec, which, device)
        broadcast_bytes(t, 0, group)
        torch.cuda.synchronize(device)
        if rank != 0:
            dec.adopt_arena(which)


def max_over_ranks(value: float, device=None, group=None) -> float:
    """The maximum of a per-rank scalar (e.g. elapsed device time)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64,
                     device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


FRAME_BYTES = 3 * 512 * 512 * 4  # one decoded frame, float32 CHW


def pipeline_plan(n_frames: int, world: int, chunk: int = 50) -> list[list[tuple[int, int]]]:
    """Per sampler chunk k, the [lo, hi) frames each rank decodes when rank 0
    runs the serial stages and the decode overlaps them:

    * one rank: rank 0 decodes everything (after the sampler);
    * two ranks: rank 1 decodes the chunks as they come and rank 0 the last
      n_chunks // 7 of them once its sampler is done (one decoding GPU alone
      falls behind the sampler);
    * more ranks: each chunk is split in contiguous ranges over ranks
      1 .. world-1 whose sizes differ by at most one frame (the larger
      ranges rotate from chunk to chunk); rank 0 only samples.
    """
    if n_frames < 0 or world < 1 or chunk < 1:
        raise ValueError("bad plan arguments")
    n_chunks = -(-n_frames // chunk)
    tail = n_chunks // 7
    plan = []
    for k in range(n_chunks):
        f0, f1 = k * chunk, min(n_frames, (k + 1) * chunk)
        ranges = [(f0, f0)] * world
        if world == 1:
            ranges[0] = (f0, f1)
        elif world == 2:
            ranges[0 if k >= n_chunks - tail else 1] = (f0, f1)
        else:
            m, n = world - 1, f1 - f0
            lo = f0
            for i in range(m):
                size = n // m + (1 if (i - k) % m < n % m else 0)
                ranges[1 + i] = (lo, lo + size)
                lo += size
        plan.append(ranges)
    return plan


def frames_per_rank(plan: list[list[tuple[int, int]]], rank: int) -> int:
    return sum(hi - lo for ranges in plan for lo, hi in (ranges[rank],))


def generate_pipelined(rank: int, world: int, device, n_frames: int, dec, frames, pipe=None, image=None,
                       audio=None, emotion: int = 0, seed: int = 0, noise=None, group=None,
                       chunk: int = 50) -> int:
    """Config-4 generation on `world` GPUs with the decode overlapping the
    sampler (pipeline_plan). Rank 0 passes `pipe` (a tpmd.Pipeline whose
    decoder is `dec`) and the inputs; the other ranks pass a MotionDecoder
    that already holds rank 0's weight arena (share_decoder or
    adopt_arena(0)). Every rank writes the frames it decodes, in frame order,
    into `frames` (host float32 [m, 3, 512, 512], m >= its frame count;
    pinned for full copy speed). Returns the number of frames this rank
    decoded. Every rank takes the same collective steps: one feats broadcast
    and one styles broadcast per chunk."""
    import numpy as np
    import torch

    plan = pipeline_plan(n_frames, world, chunk)
    n_chunks = len(plan)
    fbytes = FRAME_BYTES
    out = frames.data_ptr()
    st_dev = torch.empty((max(n_chunks, 1), chunk, 512), dtype=torch.float32, device=device)
    done = 0
    if rank == 0:
        own = []

        def on_chunk(f0, styles):
            k = f0 // chunk
            if world > 1:
                if k == 0:
                    broadcast_bytes(arena_tensor(dec, 1, device), 0, group)
                st_dev[k, :styles.shape[0]].copy_(torch.from_numpy(styles))
                broadcast_bytes(st_dev[k], 0, group)
            lo, hi = plan[k][0]
            if hi > lo:
                own.append(styles[lo - f0:hi - f0].copy())
            return 0

        pipe.styles_cb(image, audio, emotion, on_chunk, noise=noise, seed=seed)
        if own:
            st = np.ascontiguousarray(np.concatenate(own))
            dec.decode_ptr(st.ctypes.data, st.shape[0], out)
            done = st.shape[0]
    else:
        for k in range(n_chunks):
            if k == 0:
                broadcast_bytes(arena_tensor(dec, 1, device), 0, group)
                if torch.device(device).type == "cuda":
                    torch.cuda.synchronize(device)
                dec.adopt_arena(1)
            broadcast_bytes(st_dev[k], 0, group)
            lo, hi = plan[k][rank]
            if hi > lo:
                f0 = k * chunk
                s_h = st_dev[k, lo - f0:hi - f0].cpu()
                dec.decode_ptr(s_h.data_ptr(), hi - lo, out + done * fbytes)
                done += hi - lo
    return done
