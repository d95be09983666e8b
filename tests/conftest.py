"""Shared fixtures. `gpu`-marked tests need an sm_100 GPU and run the CUDA
path through the C ABI; everything else runs on CPU."""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "talking-portrait.cpp_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def golden():
    d = np.load(os.path.join(ROOT, "tests", "golden", "ops_golden.npz"))
    meta = json.loads(bytes(d["meta"]).decode())
    return d, meta


def _model(flow_gain):
    from tpmd import synth
    import oracle as O
    raw = synth.make_weights(seed=0, bias_std=0.1, flow_gain=flow_gain)
    w = synth.fold(raw, O.scale_for)
    feats = synth.make_feats(seed=0)
    styles = synth.styles_config0(seed=0, n=4)
    return dict(raw=raw, w=w, feats=feats, styles=styles)


@pytest.fixture(scope="session")
def model():
    """The parity configuration: folded random-init weights (biases
    N(0, 0.1) so bias paths count, ToFlow gain PARITY_FLOW_GAIN), smooth
    feats, a few config-0 styles."""
    from tpmd import synth
    return _model(synth.PARITY_FLOW_GAIN)


@pytest.fixture(scope="session")
def stress_model():
    """plain random init (ToFlow gain 1): the chaotic stress configuration"""
    return _model(1.0)


@pytest.fixture(scope="session")
def oracle_dec(model):
    import oracle as O
    return O.Decoder(model["w"], model["feats"])


@pytest.fixture(scope="session")
def oracle_frames(model, oracle_dec):
    """exact-graph fp32 oracle frames of model['styles'] (cached)"""
    return np.stack([oracle_dec.decode(s, mode=0) for s in model["styles"]])


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] == 10
    except Exception:
        return False
