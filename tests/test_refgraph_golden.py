"""The oracle against golden outputs of the reference's own decoder and
encoder (tests/golden/refgraph_golden.npz, written by
tests/golden/make_refgraph_golden.py from oracle/_ref's build of the
reference's src/motion_dec.cpp, src/motion_enc.cpp and src/gguf_load.cpp).
Runs without the reference tree: the inputs are regenerated from their
seeds and the oracle's outputs are summarised the same way (strided sample,
128 chunk sums, L2 norm).

Tolerances as in test_refgraph.py: f32 graphs 1 - cosine <= 1e-8 on the
sample, the reference's f16 fast graph against the oracle's emulation of it
1 - cosine <= 3e-5."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

import oracle as O
from metrics import cosine

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "refgraph_golden.npz")
sys.path.insert(0, os.path.dirname(GOLDEN))
import make_refgraph_golden as mg  # noqa: E402


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


def _summ(x):
    return mg.summarize(x)


def _check(gold, key, x, tol):
    s = _summ(x)
    a, b = s["sample"], gold[f"{key}/sample"]
    assert a.shape == b.shape, key
    d = 1.0 - cosine(a, b)
    cs, cg = s["chunks"], gold[f"{key}/chunks"]
    cd = float(np.max(np.abs(cs - cg)) / (np.max(np.abs(cg)) + 1e-30))
    nd = float(abs(s["norm"][0] - gold[f"{key}/norm"][0]) / gold[f"{key}/norm"][0])
    assert d <= tol and cd <= max(1e-5, 300 * tol) and nd <= max(1e-6, 30 * tol), (key, d, cd, nd)
    return d


@pytest.fixture(scope="module")
def inputs():
    from tpmd import synth
    raw = synth.make_weights(seed=0, bias_std=0.1, flow_gain=synth.PARITY_FLOW_GAIN)
    return dict(raw=raw, feats=synth.make_feats(seed=0), styles=synth.styles_config0(seed=0, n=2))


def test_exact_graph_against_reference_golden(gold, inputs):
    from tpmd import synth
    od = O.Decoder(synth.fold(inputs["raw"], O.scale_for), inputs["feats"])
    img = od.decode(inputs["styles"][0], mode=0, keep_taps=True)
    worst = _check(gold, "exact/img", img, 1e-8)
    for j in range(7):
        for k in ("conv1", "conv2", "flowmap", "out", "rgb"):
            worst = max(worst, _check(gold, f"exact/r{8 << j}.{k}", od.tap(f"r{8 << j}.{k}"), 1e-8))
    print(f"exact graph vs reference golden: worst 1-cos {worst:.2e}")


def test_fast_graphs_against_reference_golden(gold, inputs):
    from tpmd import synth
    od = O.Decoder(synth.fold(inputs["raw"], O.scale_for), inputs["feats"])
    raw16 = {k: v.astype(np.float16).astype(np.float32) for k, v in inputs["raw"].items()}
    od16 = O.Decoder(synth.fold(raw16, O.scale_for), inputs["feats"])
    for i, st in enumerate(inputs["styles"]):
        d32 = _check(gold, f"fast32/img{i}", od.decode(st, mode=1), 1e-8)
        d16 = _check(gold, f"fast16/img{i}", od16.decode(st, mode=1 | O.REF_F16_GRAPH), 3e-5)
        print(f"frame {i}: fast f32 1-cos {d32:.2e}; fast f16 1-cos {d16:.2e}")


def test_encoder_against_reference_golden(gold):
    from tpmd import synth
    o = O.Encoder(synth.fold(synth.make_encoder_weights(0), O.scale_for)).run(synth.make_image(0))
    for k in ("appearance", "lam", "motion"):
        assert 1.0 - cosine(o[k], gold[f"enc/{k}"]) <= 1e-9, k
    for j in range(7):
        _check(gold, f"enc/feat{j}", o["feats"][j], 1e-9)
