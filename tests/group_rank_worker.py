"""One rank of tests/test_gpu_group.py's two-process group (a test helper,
run as a child process): rank r uses GPU r, joins the clique with the id
the parent wrote, receives the weights and feats from rank 0, decodes its
shard of the styles into the whole-clip buffer and saves it."""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (os.path.join(ROOT, "talking-portrait.cpp_b200"), os.path.join(ROOT, "oracle"), HERE):
    sys.path.insert(0, p)


def main() -> int:
    import tpmd
    from conftest import _model
    from tpmd import synth
    rank, nranks, d = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3]
    nccl_id = open(os.path.join(d, "id.bin"), "rb").read()
    g = tpmd.MotionDecoderGroup((rank,), tpmd.DTYPE_F16, 4, rank=rank, nranks=nranks, nccl_id=nccl_id)
    if rank == 0:
        m = _model(synth.PARITY_FLOW_GAIN)
        g.set_tensors(m["w"])
    g.prepare()
    g.set_feats(m["feats"] if rank == 0 else None)
    st = np.load(os.path.join(d, "styles.npy"))
    out = g.decode(st)
    np.save(os.path.join(d, f"frames{rank}.npy"), out)
    np.save(os.path.join(d, f"max{rank}.npy"), np.array(g.max(float(rank))))
    g.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
