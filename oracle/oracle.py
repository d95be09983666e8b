"""ctypes bindings for the CPU oracle (liboracle.so) and, when built, the
reference's own op code (_ref/libtpref.so) and its own decoder, encoder and
weight loader over a ggml stand-in (_ref/libtpgraph.so, see RefGraph).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference legs, as the checker. The product
(libtpmd.so and its Python binding) never imports this module.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libtpref.so")
GRAPH_SO = os.path.join(HERE, "_ref", "libtpgraph.so")

# f16 emulation flags for Decoder.decode(mode=...), see tp_oracle.h
F16_WEIGHTS, F16_FEATS, F16_ACTS, F16_OUT, F16_FOLD = 0x10, 0x20, 0x40, 0x80, 0x100
REF_F16 = F16_WEIGHTS | F16_FEATS | F16_ACTS  # f16 weights, feats and conv inputs
# the reference's f16 fast graph as it runs (use with mode 1): REF_F16 plus its
# fold-into-weights rule and f16 style GEMVs (pinned against oracle/_ref's
# build of the reference's own graph)
REF_F16_GRAPH = REF_F16 | F16_FOLD

ST_IC = (512, 512, 512, 512, 256, 128, 64)
ST_OC = (512, 512, 512, 256, 128, 64, 32)

_f32p = C.POINTER(C.c_float)
_i64p = C.POINTER(C.c_int64)


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def build() -> None:
    """Compile liboracle.so (and oracle/_ref when the reference is present)."""
    import subprocess
    import sys
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    subprocess.run([sys.executable, os.path.join(HERE, "ref_build.py")], check=True)


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = C.CDLL(ORACLE_SO)
        v = C.c_void_p
        L.orc_bilinear_gather.argtypes = [v, C.c_int, C.c_int, C.c_int, C.c_int, v, C.c_int64,
                                          C.c_int, C.c_int, v]
        L.orc_im2col_cf.argtypes = [v] + [C.c_int] * 12 + [v, C.c_int]
        L.orc_bias_lrelu.argtypes = [v, v, v, C.c_int, C.c_float, v]
        L.orc_subpix_lrelu.argtypes = [v, v, v, C.c_int, C.c_int, C.c_int, C.c_float, v]
        L.orc_subpix_lrelu_cl.argtypes = [v, v, C.c_int, C.c_int64, C.c_int64, C.c_int,
                                          C.c_float, v]
        L.orc_upfirdn2x.argtypes = [v, v, C.c_int, C.c_int, C.c_int64, v]
        L.orc_blur.argtypes = [v, v, C.c_int, C.c_int, C.c_int64, C.c_int, C.c_int, v]
        L.orc_clsp_mul.argtypes = [v, v, C.c_int, C.c_int64, v]
        L.orc_clsp_lerp.argtypes = [v, v, v, C.c_int, C.c_int64, v]
        L.orc_flow_grid.argtypes = [v, v, C.c_int64, v]
        L.orc_scale_for.argtypes = [C.c_char_p, v]
        L.orc_scale_for.restype = C.c_double
        L.orc_saug.argtypes = [v, C.c_int, C.c_int, v]
        L.orc_tsubcf.argtypes = [v, v, C.c_int, C.c_int, v]
        L.orc_dec_create.restype = v
        L.orc_dec_destroy.argtypes = [v]
        L.orc_dec_set.argtypes = [v, C.c_char_p, v, C.c_int64]
        L.orc_dec_set_feat.argtypes = [v, C.c_int, v, C.c_int64]
        L.orc_dec_prepare.argtypes = [v]
        L.orc_dec_decode.argtypes = [v, v, C.c_int, C.c_int, v]
        L.orc_dec_tap.argtypes = [v, C.c_char_p, v, C.c_int64]
        L.orc_dec_tap.restype = C.c_int64
        L.orc_dec_error.argtypes = [v]
        L.orc_dec_error.restype = C.c_char_p
        L.orc_enc_create.restype = v
        L.orc_enc_destroy.argtypes = [v]
        L.orc_enc_set.argtypes = [v, C.c_char_p, v, C.c_int64]
        L.orc_enc_run.argtypes = [v, v, v, v, v, C.POINTER(v)]
        L.orc_enc_error.argtypes = [v]
        L.orc_enc_error.restype = C.c_char_p
        L.orc_fmt_create.argtypes = [v]
        L.orc_fmt_create.restype = v
        L.orc_fmt_destroy.argtypes = [v]
        L.orc_fmt_set.argtypes = [v, C.c_char_p, v, C.c_int64]
        L.orc_fmt_forward.argtypes = [v, v, v, C.c_float, v]
        L.orc_fmt_sample.argtypes = [v, v, v, v, v, v, C.c_int, v]
        L.orc_fmt_error.argtypes = [v]
        L.orc_fmt_error.restype = C.c_char_p
        L.orc_aud_create.argtypes = [v]
        L.orc_aud_create.restype = v
        L.orc_aud_destroy.argtypes = [v]
        L.orc_aud_set.argtypes = [v, C.c_char_p, v, C.c_int64]
        L.orc_aud_encode.argtypes = [v, v, C.c_int64, C.c_int64, v]
        L.orc_aud_error.argtypes = [v]
        L.orc_aud_error.restype = C.c_char_p
        L.orc_chw_to_rgb24.argtypes = [v, C.c_int64, C.c_int64, v]
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_get_threads.restype = C.c_int
        _lib = L
    return _lib


def ref_lib():
    """The reference's op code built by ref_build.py, or None if absent."""
    global _ref
    if _ref is None and os.path.exists(REF_SO):
        L = C.CDLL(REF_SO)
        v = C.c_void_p
        for pre in ("ref_cpu_", "ref_cu_"):
            getattr(L, pre + "bilinear_gather").argtypes = [v, C.c_int, C.c_int, C.c_int, C.c_int,
                                                           v, C.c_int64, C.c_int, C.c_int, v]
            getattr(L, pre + "bias_lrelu").argtypes = [v, v, v, C.c_int, C.c_float, v]
            getattr(L, pre + "subpix_lrelu").argtypes = [v, v, v, C.c_int, C.c_int, C.c_int,
                                                        C.c_float, v]
            getattr(L, pre + "subpix_lrelu_cl").argtypes = [v, v, C.c_int, C.c_int64, C.c_int64,
                                                           C.c_int, C.c_float, v]
            getattr(L, pre + "upfirdn2x").argtypes = [v, v, C.c_int, C.c_int, C.c_int64, v]
            getattr(L, pre + "flow_grid").argtypes = [v, v, C.c_int64, v]
        L.ref_cpu_clsp_mul.argtypes = [v, v, C.c_int, C.c_int64, v]
        L.ref_cpu_clsp_lerp.argtypes = [v, v, v, C.c_int, C.c_int64, v]
        L.ref_cu_clsp.argtypes = [v, v, v, C.c_int, C.c_int64, C.c_int, v]
        L.ref_cu_im2col_cf.argtypes = [v] + [C.c_int] * 12 + [v, C.c_int]
        _ref = L
    return _ref


# ---------------------------------------------------------------------------
# op wrappers. `impl` selects: "oracle" (this restatement), "ref_cpu" or
# "ref_cu" (the reference's own CPU function / CUDA kernel run on the host).
# ---------------------------------------------------------------------------
def _L(impl):
    if impl == "oracle":
        return lib(), "orc_"
    r = ref_lib()
    if r is None:
        raise RuntimeError("oracle/_ref/libtpref.so not built (reference absent)")
    return r, impl + "_"


def bilinear_gather(feat, W, H, grid, planar=False, sp=False, impl="oracle"):
    feat = np.ascontiguousarray(feat)
    grid = np.ascontiguousarray(grid, dtype=np.float32)
    Cc = feat.shape[-1]
    N = grid.size // 2
    out = np.empty((Cc, N) if sp else (N, Cc), np.float32)
    L, pre = _L(impl)
    getattr(L, pre + "bilinear_gather")(_p(feat), int(feat.dtype == np.float16), Cc, W, H,
                                        _p(grid), N, int(planar), int(sp), _p(out))
    return out


def im2col_cf(src, IC, IW, IH, N, KW=3, KH=3, s0=1, s1=1, p0=1, p1=1, d0=1, d1=1,
              dst_f16=False, impl="oracle"):
    src = np.ascontiguousarray(src, dtype=np.float32)
    OW = (IW + 2 * p0 - d0 * (KW - 1) - 1) // s0 + 1
    OH = (IH + 2 * p1 - d1 * (KH - 1) - 1) // s1 + 1
    out = np.empty((N, OH, OW, IC * KW * KH), np.float16 if dst_f16 else np.float32)
    if impl == "oracle":
        lib().orc_im2col_cf(_p(src), IC, IW, IH, N, KW, KH, s0, s1, p0, p1, d0, d1, _p(out),
                            int(dst_f16))
    else:
        if impl != "ref_cu":
            raise ValueError("im2col_cf reference: only the CUDA kernel is self-contained")
        _L(impl)[0].ref_cu_im2col_cf(_p(src), IC, IW, IH, N, KW, KH, s0, s1, p0, p1, d0, d1,
                                     _p(out), int(dst_f16))
    return out


def bias_lrelu(x, bias, axis, slope=0.2, impl="oracle"):
    """x given in ggml ne order as a flat array plus ne (4-tuple)."""
    arr, ne = x
    arr = np.ascontiguousarray(arr, np.float32)
    ne = np.asarray(list(ne) + [1] * (4 - len(ne)), np.int64)
    bias = np.ascontiguousarray(bias, np.float32)
    out = np.empty_like(arr)
    L, pre = _L(impl)
    getattr(L, pre + "bias_lrelu")(_p(arr), _p(bias), _p(ne), axis, slope, _p(out))
    return out


def subpix_lrelu(g0, g1, bias, W, H, OC, slope=0.2, impl="oracle"):
    out = np.empty(4 * W * H * OC, np.float32)
    L, pre = _L(impl)
    getattr(L, pre + "subpix_lrelu")(_p(g0), _p(g1), _p(bias), W, H, OC, slope, _p(out))
    return out


def subpix_lrelu_cl(y4, bias, OC, N, B, W, slope=0.2, impl="oracle"):
    out = np.empty(4 * OC * N * B, np.float32)
    L, pre = _L(impl)
    getattr(L, pre + "subpix_lrelu_cl")(_p(y4), _p(bias), OC, N, B, W, slope, _p(out))
    return out


def upfirdn2x(x, k4, W, H, CB, impl="oracle"):
    out = np.empty(4 * W * H * CB, np.float32)
    L, pre = _L(impl)
    getattr(L, pre + "upfirdn2x")(_p(x), _p(k4), W, H, CB, _p(out))
    return out


def blur(x, k4, W, H, Cc, p0, p1):
    """oracle Blur: x [C][H][W] -> [C][H+p0+p1-3][W+p0+p1-3]"""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty((Cc, H + p0 + p1 - 3, W + p0 + p1 - 3), np.float32)
    lib().orc_blur(_p(x), _p(np.ascontiguousarray(k4, np.float32)), W, H, Cc, p0, p1, _p(out))
    return out


def clsp(cl, m, Cc, N, o=None, impl="oracle"):
    out = np.empty(Cc * N, np.float32)
    L, pre = _L(impl)
    if impl == "ref_cu":
        L.ref_cu_clsp(_p(cl), _p(m), _p(o) if o is not None else None, Cc, N,
                      int(o is not None), _p(out))
    elif o is None:
        getattr(L, pre + "clsp_mul")(_p(cl), _p(m), Cc, N, _p(out))
    else:
        getattr(L, pre + "clsp_lerp")(_p(cl), _p(m), _p(o), Cc, N, _p(out))
    return out


def flow_grid(fl, xs, N, impl="oracle"):
    out = np.empty(3 * N, np.float32)
    L, pre = _L(impl)
    getattr(L, pre + "flow_grid")(_p(fl), _p(xs), N, _p(out))
    return out


def scale_for(name: str, ne) -> float:
    ne = np.asarray(list(ne) + [1] * (4 - len(ne)), np.int64)
    return lib().orc_scale_for(name.encode(), _p(ne))


def saug(W, IC, OC):
    out = np.empty((OC, IC + 1), np.float32)
    lib().orc_saug(_p(np.ascontiguousarray(W, np.float32)), IC, OC, _p(out))
    return out


def tsubcf(W, K, IC, OC):
    out = np.empty((4 * OC, 9 * IC), np.float32)
    lib().orc_tsubcf(_p(np.ascontiguousarray(W, np.float32)),
                     _p(np.ascontiguousarray(K, np.float32)), IC, OC, _p(out))
    return out


class Decoder:
    """The oracle decoder: folded tensors in, CHW f32 frames out."""

    def __init__(self, tensors: dict, feats: list):
        L = lib()
        self._L = L
        self._h = L.orc_dec_create()
        for name, arr in tensors.items():
            a = np.ascontiguousarray(arr, np.float32)
            if L.orc_dec_set(self._h, name.encode(), _p(a), a.size) != 0:
                raise ValueError(self.error())
        for j, f in enumerate(feats):
            a = np.ascontiguousarray(f, np.float32)
            if L.orc_dec_set_feat(self._h, j, _p(a), a.size) != 0:
                raise ValueError(self.error())
        if L.orc_dec_prepare(self._h) != 0:
            raise ValueError(self.error())

    def error(self) -> str:
        return self._L.orc_dec_error(self._h).decode()

    def decode(self, style, mode=0, keep_taps=False):
        style = np.ascontiguousarray(style, np.float32)
        img = np.empty((3, 512, 512), np.float32)
        if self._L.orc_dec_decode(self._h, _p(style), mode, int(keep_taps), _p(img)) != 0:
            raise RuntimeError(self.error())
        return img

    def tap(self, name: str) -> np.ndarray:
        n = self._L.orc_dec_tap(self._h, name.encode(), None, 0)
        if n < 0:
            raise KeyError(name)
        out = np.empty(n, np.float32)
        self._L.orc_dec_tap(self._h, name.encode(), _p(out), n)
        return out

    def __del__(self):
        if getattr(self, "_h", None):
            self._L.orc_dec_destroy(self._h)
            self._h = None


class Encoder:
    """The motion encoder restatement (motion_enc::run, src/motion_enc.cpp:46-184)
    over scale-folded host tensors (enc.* and dec.direction.Q)."""

    def __init__(self, tensors: dict):
        self._L = lib()
        self._h = self._L.orc_enc_create()
        for n, a in tensors.items():
            a = np.ascontiguousarray(a, np.float32)
            if self._L.orc_enc_set(self._h, n.encode(), _p(a), a.size) != 0:
                raise RuntimeError(self._L.orc_enc_error(self._h).decode())

    def run(self, image: np.ndarray) -> dict:
        img = np.ascontiguousarray(image, np.float32)
        app, lam, mot = np.empty(512, np.float32), np.empty(20, np.float32), np.empty(512, np.float32)
        feats = [np.empty(((8 << j) ** 2, ST_OC[j]), np.float32) for j in range(7)]
        ptrs = (C.c_void_p * 7)(*[f.ctypes.data for f in feats])
        if self._L.orc_enc_run(self._h, _p(img), _p(app), _p(lam), _p(mot), ptrs) != 0:
            raise RuntimeError(self._L.orc_enc_error(self._h).decode())
        return dict(appearance=app, lam=lam, motion=mot, feats=feats)

    def __del__(self):
        if getattr(self, "_h", None):
            self._L.orc_enc_destroy(self._h)
            self._h = None


class FmtConfig(C.Structure):
    """orc_fmt_config: the FMT's float.fmt.* hyper-parameters."""
    _fields_ = [(n, C.c_int) for n in ("dim_h", "depth", "n_heads", "dim_w", "dim_a", "dim_e",
                                       "chunk_frames", "prev_frames", "attn_window", "t_freq_dim", "nfe")] + \
               [(n, C.c_float) for n in ("mlp_ratio", "ln_eps", "a_cfg", "e_cfg")]


class Fmt:
    """The flow-matching transformer restatement (src/fmt.cpp:9-211) and its
    chunk sampler (src/pipeline.cpp:15-91), f32."""

    def __init__(self, cfg: dict, tensors: dict):
        self._L = lib()
        self.cfg = FmtConfig(**cfg)
        self._h = self._L.orc_fmt_create(C.byref(self.cfg))
        for n, a in tensors.items():
            a = np.ascontiguousarray(a, np.float32)
            if self._L.orc_fmt_set(self._h, n.encode(), _p(a), a.size) != 0:
                raise RuntimeError(self._L.orc_fmt_error(self._h).decode())

    def forward(self, x60, cond, t: float) -> np.ndarray:
        c = self.cfg
        T = c.chunk_frames + c.prev_frames
        x60 = np.ascontiguousarray(x60, np.float32)
        cond = np.ascontiguousarray(cond, np.float32)
        v = np.empty((3, T, c.dim_w), np.float32)
        if self._L.orc_fmt_forward(self._h, _p(x60), _p(cond), float(t), _p(v)) != 0:
            raise RuntimeError(self._L.orc_fmt_error(self._h).decode())
        return v

    def sample(self, wr, prev_wa, cond_audio, prev_x, x0, emotion: int) -> np.ndarray:
        c = self.cfg
        a = [np.ascontiguousarray(z, np.float32) for z in (wr, prev_wa, cond_audio, prev_x, x0)]
        out = np.empty((c.chunk_frames, c.dim_w), np.float32)
        if self._L.orc_fmt_sample(self._h, *[_p(z) for z in a], int(emotion), _p(out)) != 0:
            raise RuntimeError(self._L.orc_fmt_error(self._h).decode())
        return out

    def __del__(self):
        if getattr(self, "_h", None):
            self._L.orc_fmt_destroy(self._h)
            self._h = None


class AudConfig(C.Structure):
    """orc_aud_config: the audio encoder's float.audio.* hyper-parameters."""
    _fields_ = [("n_layers", C.c_int), ("n_heads", C.c_int), ("hidden", C.c_int), ("ffn", C.c_int),
                ("dim_w", C.c_int), ("ln_eps", C.c_float), ("conv_dim", C.c_int * 7),
                ("conv_kernel", C.c_int * 7), ("conv_stride", C.c_int * 7), ("pos_kernel", C.c_int),
                ("pos_groups", C.c_int), ("sample_rate", C.c_int), ("fps", C.c_int)]


def aud_config(cfg: dict) -> AudConfig:
    c = AudConfig()
    for k, val in cfg.items():
        if k.startswith("conv_"):
            getattr(c, k)[:] = list(val)
        else:
            setattr(c, k, val)
    return c


class Aud:
    """The audio encoder restatement (audio_model::encode, src/audio_enc.cpp:55-236), f32."""

    def __init__(self, cfg: dict, tensors: dict):
        self._L = lib()
        self.cfg = dict(cfg)
        self._c = aud_config(cfg)
        self._h = self._L.orc_aud_create(C.byref(self._c))
        for n, a in tensors.items():
            a = np.ascontiguousarray(a, np.float32)
            if self._L.orc_aud_set(self._h, n.encode(), _p(a), a.size) != 0:
                raise RuntimeError(self._L.orc_aud_error(self._h).decode())

    def encode(self, audio, seq_len: int) -> np.ndarray:
        a = np.ascontiguousarray(audio, np.float32)
        out = np.empty((seq_len, self.cfg["dim_w"]), np.float32)
        if self._L.orc_aud_encode(self._h, _p(a), a.size, seq_len, _p(out)) != 0:
            raise RuntimeError(self._L.orc_aud_error(self._h).decode())
        return out

    def __del__(self):
        if getattr(self, "_h", None):
            self._L.orc_aud_destroy(self._h)
            self._h = None


def chw_to_rgb24(frames) -> np.ndarray:
    """[n][3][H][W] f32 -> [n][H][W][3] uint8, tools/tp-cli.cpp:43-53"""
    f = np.ascontiguousarray(frames, np.float32)
    n, c, h, w = f.shape
    out = np.empty((n, h, w, 3), np.uint8)
    lib().orc_chw_to_rgb24(_p(f), n, h * w, _p(out))
    return out


def set_threads(n: int) -> None:
    lib().orc_set_threads(n)


def threads() -> int:
    return lib().orc_get_threads()


_graph = None


def graph_lib():
    """oracle/_ref/libtpgraph.so (built by ref_build.py), or None if absent."""
    global _graph
    if _graph is None and os.path.exists(GRAPH_SO):
        L = C.CDLL(GRAPH_SO)
        v = C.c_void_p
        L.rg_create.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_char_p, C.c_size_t]
        L.rg_create.restype = v
        L.rg_destroy.argtypes = [v]
        L.rg_error.argtypes = [v]
        L.rg_error.restype = C.c_char_p
        L.rg_tensor.argtypes = [v, C.c_char_p, v, C.c_int64]
        L.rg_tensor.restype = C.c_int64
        L.rg_build.argtypes = [v, C.c_int, C.c_int, C.c_int]
        L.rg_batch.argtypes = [v]
        L.rg_set_feats.argtypes = [v, C.POINTER(v)]
        L.rg_decode.argtypes = [v, v, v, C.c_int]
        L.rg_decode_batch.argtypes = [v, v, v]
        L.rg_tap.argtypes = [v, C.c_char_p, v, C.c_int64]
        L.rg_tap.restype = C.c_int64
        L.rg_enc_run.argtypes = [v, v, v, v, v, C.POINTER(v), C.c_int]
        _graph = L
    return _graph


class RefGraph:
    """The reference's own motion_ae path run on the CPU: weights_t::load of a
    GGUF file (src/gguf_load.cpp) with motion_ae_scale (src/motion_enc.cpp),
    motion_dec::prepare / build / set_feats / decode / decode_batch
    (src/motion_dec.cpp) and motion_enc::run, compiled from the reference's
    sources over the stand-in in oracle/refgraph/. keep_f16 is the
    reference's f16 fast path (tp_ctx::load with ftype "f16")."""

    def __init__(self, gguf_path: str, keep_f16: bool = False, gpu: bool = False):
        L = graph_lib()
        if L is None:
            raise RuntimeError("oracle/_ref/libtpgraph.so not built (reference absent)")
        self._L = L
        err = C.create_string_buffer(512)
        self._h = L.rg_create(gguf_path.encode(), int(keep_f16), int(gpu), err, len(err))
        if not self._h:
            raise RuntimeError(err.value.decode())

    def _ck(self, rc):
        if rc != 0:
            raise RuntimeError(self._L.rg_error(self._h).decode())

    def tensor(self, name: str) -> np.ndarray:
        """a loaded weight or a prepare()-derived tensor, f32, ggml order"""
        n = self._L.rg_tensor(self._h, name.encode(), None, 0)
        if n < 0:
            raise KeyError(name)
        out = np.empty(n, np.float32)
        self._L.rg_tensor(self._h, name.encode(), _p(out), n)
        return out

    def build(self, taps: bool = False, batch: int = 1, stages: int = 7) -> int:
        """stages < 7: the graph ends at that stage and its image is the rgb
        skip [3][r][r] of stage r = 8 << (stages - 1)"""
        self._ck(self._L.rg_build(self._h, int(taps), batch, stages))
        self.stages = stages
        return self._L.rg_batch(self._h)

    def set_feats(self, feats):
        arrs = [np.ascontiguousarray(f, np.float32) for f in feats]
        self._keep = arrs
        self._ck(self._L.rg_set_feats(self._h, (C.c_void_p * 7)(*[a.ctypes.data for a in arrs])))

    def decode(self, style, taps: bool = False) -> np.ndarray:
        st = np.ascontiguousarray(style, np.float32)
        img = np.empty((3, 512, 512), np.float32)
        self._ck(self._L.rg_decode(self._h, _p(st), _p(img), int(taps)))
        return img

    def decode_batch(self, styles) -> np.ndarray:
        st = np.ascontiguousarray(styles, np.float32)
        out = np.empty((st.shape[0], 3, 512, 512), np.float32)
        self._ck(self._L.rg_decode_batch(self._h, _p(st), _p(out)))
        return out

    def tap(self, name: str) -> np.ndarray:
        n = self._L.rg_tap(self._h, name.encode(), None, 0)
        if n < 0:
            raise KeyError(name)
        out = np.empty(n, np.float32)
        self._L.rg_tap(self._h, name.encode(), _p(out), n)
        return out

    def encode(self, image, taps: bool = False) -> dict:
        img = np.ascontiguousarray(image, np.float32)
        app, lam, mot = np.empty(512, np.float32), np.empty(20, np.float32), np.empty(512, np.float32)
        feats = [np.empty(((8 << j) ** 2, ST_OC[j]), np.float32) for j in range(7)]
        ptrs = (C.c_void_p * 7)(*[f.ctypes.data for f in feats])
        self._ck(self._L.rg_enc_run(self._h, _p(img), _p(app), _p(lam), _p(mot), ptrs, int(taps)))
        return dict(appearance=app, lam=lam, motion=mot, feats=feats)

    def __del__(self):
        if getattr(self, "_h", None):
            self._L.rg_destroy(self._h)
            self._h = None
