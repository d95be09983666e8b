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

The reference has no multi-GPU path (src/pipeline.cpp:153-184 decodes
batches serially on one device); this module is new.
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
