"""The GGUF v3 reader (tpmd_gguf_read / tpmd_gguf_read_kv, host code) on
corrupted files: the input-only robustness the reference checks with its
libFuzzer targets. Seeded mutations of a small valid file (byte flips,
truncations, inserted and deleted bytes, and counts, lengths, ranks,
dimensions and offsets set to huge or boundary values) must each read or
fail with an error, never crash or hang. The reads run in a child process,
so a crash shows up as its exit status (with the last file it reached)."""
from __future__ import annotations

import os
import struct
import subprocess
import sys

import numpy as np

import gguf_writer as gw

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

CHILD = r"""
import sys
sys.path.insert(0, sys.argv[1])
import tpmd
ok = err = 0
for i, path in enumerate(sys.argv[2:]):
    print(i, flush=True)
    for fn in (lambda: tpmd.gguf_read(path, None, fold=False),
               lambda: tpmd.gguf_read(path, "float-motion-ae", fold=True),
               lambda: tpmd.gguf_kv(path)):
        try:
            fn()
            ok += 1
        except (tpmd.TpmdError, ValueError, RuntimeError):
            err += 1
print("done", ok, err, flush=True)
"""


def _base(path):
    rng = np.random.default_rng(3)
    gw.write(path, [("dec.conv1.conv.weight", rng.standard_normal((1, 4, 2, 3, 3)).astype(np.float32), "f32"),
                    ("dec.convs.0.activate.bias", rng.standard_normal(4).astype(np.float32), "f16"),
                    ("dec.x", np.ones((2, 3), np.float32), "f32")],
             extra_kv=[("float.n", gw.T_U32, 7), ("float.s", gw.T_STR, "abc"), ("float.f", gw.T_F32, 0.5)])
    return open(path, "rb").read()


def _mutants(data: bytes, n: int, seed: int):
    rng = np.random.default_rng(seed)
    huge = [0, 1, 2**31 - 1, 2**31, 2**32 - 1, 2**32, 2**62, 2**63 - 1, 2**64 - 1]
    out = []
    for _ in range(n):
        b = bytearray(data)
        kind = int(rng.integers(0, 6))
        if kind == 0:  # flip a few bytes
            for _ in range(int(rng.integers(1, 6))):
                b[int(rng.integers(0, len(b)))] ^= int(rng.integers(1, 256))
        elif kind == 1:  # truncate
            b = b[:int(rng.integers(0, len(b)))]
        elif kind == 2:  # insert bytes
            at = int(rng.integers(0, len(b)))
            b[at:at] = bytes(rng.integers(0, 256, int(rng.integers(1, 16)), dtype=np.uint8))
        elif kind == 3:  # delete bytes
            at = int(rng.integers(0, len(b)))
            del b[at:at + int(rng.integers(1, 16))]
        else:  # a 4- or 8-byte field in the header / KV / tensor-info region set to a boundary value
            w = 8 if kind == 4 else 4
            at = int(rng.integers(0, min(len(b), 400) - w))
            v = huge[int(rng.integers(0, len(huge)))] & ((1 << (8 * w)) - 1)
            b[at:at + w] = v.to_bytes(w, "little")
        out.append(bytes(b))
    # the header's counts themselves at boundary values
    for off in (8, 16):  # n_tensors, n_kv
        for v in huge:
            b = bytearray(data)
            b[off:off + 8] = struct.pack("<Q", v)
            out.append(bytes(b))
    return out


def test_corrupted_files_fail_cleanly(tmp_path):
    data = _base(str(tmp_path / "base.gguf"))
    paths = []
    for i, m in enumerate(_mutants(data, 2000, seed=11)):
        p = str(tmp_path / f"m{i:04d}.gguf")
        with open(p, "wb") as f:
            f.write(m)
        paths.append(p)
    pkg = os.path.join(ROOT, "talking-portrait.cpp_b200")
    for lo in range(0, len(paths), 200):
        batch = paths[lo:lo + 200]
        r = subprocess.run([sys.executable, "-c", CHILD, pkg] + batch, capture_output=True, text=True,
                           timeout=300)
        last = r.stdout.strip().splitlines()[-1] if r.stdout.strip() else "(none)"
        assert r.returncode == 0, f"reader crashed (exit {r.returncode}) after file index {last} of batch {lo}: " \
                                  f"{r.stderr[-400:]}"
        assert last.startswith("done"), last
