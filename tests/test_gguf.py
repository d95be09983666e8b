"""GGUF v3 reader (tpmd_gguf_read / tpmd_load_gguf) against the reference
loader's behaviour (src/gguf_load.cpp:50-197): dims, f16 conversion, scale
folding, and every rejection path. CPU only: the reader needs no GPU."""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "talking-portrait.cpp_b200"))
import tpmd  # noqa: E402
from tpmd import synth  # noqa: E402

import gguf_writer as gw  # noqa: E402

ARCH = "float-motion-ae"


def _decoder_tensors(raw, dt):
    return [(n, a.reshape(gw.torch_shape(n, a.shape)), dt) for n, a in raw.items()]


def _extra_tensors(rng):
    # tensors of the same file the decoder does not take
    return [("enc.net_app.convs.0.0.weight", rng.standard_normal((8, 3, 3, 3)).astype(np.float32), "f32"),
            ("dec.direction.weight", rng.standard_normal((512, 20)).astype(np.float32), "f32")]


@pytest.fixture(scope="module")
def raw():
    return synth.make_weights(0, bias_std=0.1)


@pytest.fixture(scope="module")
def f32_file(raw, tmp_path_factory):
    p = str(tmp_path_factory.mktemp("gguf") / "motion_ae_f32.gguf")
    rng = np.random.default_rng(5)
    gw.write(p, _extra_tensors(rng) + _decoder_tensors(raw, "f32"))
    return p


def test_f32_file_reads_folded_and_exact(raw, f32_file):
    got = tpmd.gguf_read(f32_file, ARCH, fold=True)
    want = synth.fold(raw, tpmd.scale_for)
    for n, a in want.items():
        ne, v = got[n]
        assert ne == synth.ggml_ne(a.shape), n
        assert np.array_equal(v, a.reshape(-1)), n
    assert "enc.net_app.convs.0.0.weight" in got and "dec.direction.weight" in got


def test_unfolded_read_returns_file_values(raw, f32_file):
    got = tpmd.gguf_read(f32_file, None, fold=False)
    for n, a in raw.items():
        assert np.array_equal(got[n][1], a.reshape(-1).astype(np.float32)), n


def test_f16_file_converts_exactly_then_folds(raw, tmp_path):
    sub = {n: raw[n] for n in list(raw)[:12]}
    p = str(tmp_path / "motion_ae_f16.gguf")
    gw.write(p, _decoder_tensors(sub, "f16"))
    got = tpmd.gguf_read(p, ARCH, fold=True)
    want = synth.fold({n: a.astype(np.float16).astype(np.float32) for n, a in sub.items()}, tpmd.scale_for)
    for n, a in want.items():
        assert np.array_equal(got[n][1], a.reshape(-1)), n


def test_unit_dims_kept_in_order_then_dropped(tmp_path):
    p = str(tmp_path / "dims.gguf")
    gw.write(p, [("a", np.ones((1, 3, 5, 1, 1), np.float32), "f32"),     # ne [1,1,5,3,1]
                 ("b", np.ones((1, 7, 2, 3, 3), np.float32), "f32"),     # ne [3,3,2,7,1]
                 ("c", np.ones((4,), np.float32), "f32")])
    got = tpmd.gguf_read(p, None, fold=False)
    assert got["a"][0] == (1, 1, 5, 3)
    assert got["b"][0] == (3, 3, 2, 7)
    assert got["c"][0] == (4, 1, 1, 1)


def _expect_error(path, needle, arch=ARCH):
    with pytest.raises(tpmd.TpmdError, match=needle):
        tpmd.gguf_read(path, arch)


def test_rejections(tmp_path):
    t = [("dec.x", np.ones((2, 3), np.float32), "f32")]

    def f(name, **kw):
        p = str(tmp_path / name)
        gw.write(p, t if "tensors" not in kw else kw.pop("tensors"), **kw)
        return p

    _expect_error(str(tmp_path / "missing.gguf"), "cannot open")
    _expect_error(f("magic.gguf", magic=b"GGUX"), "not a GGUF file")
    _expect_error(f("v2.gguf", version=2), "unsupported GGUF version")
    _expect_error(f("arch.gguf", arch="llama"), "unexpected architecture 'llama', want float-motion-ae")
    _expect_error(f("noarch.gguf", arch=None), "unexpected architecture '<none>'")
    _expect_error(f("kv9.gguf", extra_kv=[("x.arr", gw.T_ARRAY, [1, 2])]), "unsupported KV type 9 for x.arr")
    _expect_error(f("type2.gguf", type_override={"dec.x": 2}), "tensor dec.x has unsupported type")
    _expect_error(f("oob.gguf", offset_override={"dec.x": 1 << 20}), "tensor dec.x out of bounds")
    _expect_error(f("dims.gguf", tensors=[("dec.y", np.ones((2, 2, 2, 2, 2), np.float32), "f32")]),
                  "tensor dec.y has >4 non-unit dims")
    full = f("ok.gguf")
    n = os.path.getsize(full)
    _expect_error(f("trunc_hdr.gguf", truncate=10), "corrupt header|not a GGUF|version")
    # cut inside the architecture string value (24-byte header, 28-byte key,
    # 4-byte type, 8-byte length): the KV section ends early
    _expect_error(f("trunc_kv.gguf", truncate=70), "truncated KV section")
    # cut inside the first key: like the reference's reader, the type word is
    # then read from the key's bytes and rejected as a KV type
    _expect_error(f("trunc_key.gguf", truncate=40), "unsupported KV type")
    _expect_error(f("trunc_data.gguf", truncate=n - 16), "out of bounds")  # 24 data bytes + 8 pad
    assert tpmd.gguf_read(full, ARCH)["dec.x"][1].tolist() == [1.0] * 6


def test_consumer_can_stop_the_read(f32_file):
    import ctypes as C
    L = tpmd.load_library()
    seen = []

    def cb(_u, name, ne, data, n):
        seen.append(name.decode())
        return 1 if len(seen) == 3 else 0

    err = C.create_string_buffer(256)
    rc = L.tpmd_gguf_read(f32_file.encode(), ARCH.encode(), 1, tpmd.GGUF_TENSOR_FN(cb), None, err, len(err))
    assert rc == -1 and len(seen) == 3
    assert b"rejected by the consumer" in err.value


def test_error_buffer_truncates(tmp_path):
    import ctypes as C
    L = tpmd.load_library()
    err = C.create_string_buffer(8)
    rc = L.tpmd_gguf_read(str(tmp_path / "nope.gguf").encode(), None, 1,
                          tpmd.GGUF_TENSOR_FN(lambda *a: 0), None, err, len(err))
    assert rc == -1 and len(err.value) == 7
