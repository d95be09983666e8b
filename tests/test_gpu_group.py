"""The decoder on several GPUs behind one handle (tpmd_group_*), through the
C ABI. Needs at least two GPUs (skipped otherwise): one process driving two
GPUs, and two processes with one GPU each (the torchrun layout), both
against a one-GPU decode of the same frames, bit for bit (each frame runs
the same kernels on the same bytes whichever GPU decodes it)."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

import tpmd

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _gpus():
    import torch
    return torch.cuda.device_count()


needs2 = pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")


@pytest.fixture(scope="module")
def one_gpu_frames(model):
    st = np.concatenate([model["styles"], model["styles"][:1] + 0.01])  # 5 frames
    d = tpmd.MotionDecoder(0, tpmd.DTYPE_F16, 4)
    d.set_tensors(model["w"])
    d.prepare()
    d.set_feats(model["feats"])
    return st, d.decode(st)


@needs2
def test_group_one_process_two_gpus(model, one_gpu_frames):
    st, ref = one_gpu_frames
    g = tpmd.MotionDecoderGroup((0, 1), tpmd.DTYPE_F16, 4)
    assert (g.size, g.rank0, g.nranks) == (2, 0, 2)
    g.set_tensors(model["w"])
    g.prepare()
    g.set_feats(model["feats"])
    out = g.decode(st)
    assert np.array_equal(out, ref)
    import oracle as O
    assert np.array_equal(g.decode_rgb24(st), O.chw_to_rgb24(ref))
    assert g.max(3.0) == 3.0
    g.close()


@needs2
def test_group_one_process_per_gpu(model, one_gpu_frames, tmp_path):
    st, ref = one_gpu_frames
    np.save(tmp_path / "styles.npy", st)
    nccl_id = tpmd.nccl_unique_id()
    (tmp_path / "id.bin").write_bytes(nccl_id)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TPMD_NCCL_TIMEOUT_S="60")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "group_rank_worker.py"), str(r), "2",
                               str(tmp_path)], env=env) for r in range(2)]
    rcs = [p.wait(timeout=600) for p in procs]
    assert rcs == [0, 0]
    out = np.zeros_like(ref)
    for r in range(2):
        lo, hi = tpmd.shard_range(len(st), 2, r)
        out[lo:hi] = np.load(tmp_path / f"frames{r}.npy")[lo:hi]
        assert float(np.load(tmp_path / f"max{r}.npy")) == 1.0  # max over ranks of the rank index
    assert np.array_equal(out, ref)
