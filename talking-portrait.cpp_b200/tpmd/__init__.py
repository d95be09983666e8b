"""Python binding of libtpmd.so, the B200 motion decoder's C ABI
(include/tpmd.h).

This is a thin ctypes layer: every call goes through the C ABI into the
sm_100a kernels. There is no CPU or PyTorch fallback: importing this module
without the built library raises, and the decoder refuses GPUs other than
sm_100.

Device memory for the op-level entry points and for tpmd_decode_device is
passed as torch CUDA tensors (their data_ptr) purely as the allocator; torch
computes nothing here.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import synth  # noqa: F401  (re-exported)

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(HERE), "libtpmd.so")

DTYPE_F32 = 0
DTYPE_F16 = 1
N_LEVELS = 7
STYLE_DIM = 512
IMG = 512
ST_IC = (512, 512, 512, 512, 256, 128, 64)
ST_OC = (512, 512, 512, 256, 128, 64, 32)

EXPORTS = ("tpmd_abi_version", "tpmd_create", "tpmd_create_error", "tpmd_destroy",
           "tpmd_last_error", "tpmd_scale_for", "tpmd_set_tensor", "tpmd_prepare",
           "tpmd_set_feats", "tpmd_batch", "tpmd_decode", "tpmd_decode_device",
           "tpmd_arena", "tpmd_arena_adopt", "tpmd_decode_taps", "tpmd_profile_begin", "tpmd_profile_end",
           "tpmd_kernel_launches", "tpmd_decode_noalloc", "tpmd_device_status", "tpmd_debug_expire_wait",
           "tpmd_gguf_read", "tpmd_load_gguf",
           "tpmd_set_feats_device", "tpme_create", "tpme_create_error", "tpme_destroy", "tpme_last_error",
           "tpme_set_tensor", "tpme_load_gguf", "tpme_prepare", "tpme_run", "tpme_feat_device",
           "tpmd_gguf_read_kv", "tpfm_default_config", "tpfm_create", "tpfm_create_error", "tpfm_destroy",
           "tpfm_last_error", "tpfm_set_tensor", "tpfm_load_gguf", "tpfm_prepare", "tpfm_forward",
           "tpfm_sample_chunk", "tpae_default_config", "tpae_create", "tpae_create_error", "tpae_destroy",
           "tpae_last_error", "tpae_set_tensor", "tpae_load_gguf", "tpae_prepare", "tpae_encode",
           "tppl_create", "tppl_create_error", "tppl_destroy", "tppl_last_error", "tppl_load",
           "tppl_motion_encoder", "tppl_audio_encoder", "tppl_sampler", "tppl_decoder", "tppl_prepare",
           "tppl_n_frames", "tppl_n_chunks", "tppl_generate", "tppl_generate_cb", "tppl_styles", "tppl_styles_cb",
           "tpk_bilinear_gather", "tpk_im2col_cf", "tpk_last_error",
           "tpmd_group_create", "tpmd_group_unique_id", "tpmd_group_create_rank", "tpmd_group_create_error",
           "tpmd_group_destroy", "tpmd_group_last_error", "tpmd_group_size", "tpmd_group_ranks",
           "tpmd_group_member", "tpmd_group_set_tensor", "tpmd_group_load_gguf", "tpmd_group_prepare",
           "tpmd_group_set_feats", "tpmd_group_set_feats_device", "tpmd_shard_range", "tpmd_group_decode",
           "tpmd_group_max", "tpmd_group_selftest_nccl", "tpmd_decode_rgb24", "tpmd_group_decode_rgb24",
           "tpk_chw_to_rgb24", "tpk_gemm", "tpmd_decode_schedule")

_lib = None


class TpmdError(RuntimeError):
    pass


def load_library(path: str = LIB_PATH):
    """Load libtpmd.so; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with "
                          "`python talking-portrait.cpp_b200/build.py` (no fallback exists)")
    L = C.CDLL(path)
    v, i64, cp = C.c_void_p, C.c_int64, C.c_char_p
    L.tpmd_abi_version.restype = C.c_int
    L.tpmd_create.argtypes = [C.c_int, C.c_int, C.c_int]
    L.tpmd_create.restype = v
    L.tpmd_create_error.restype = cp
    L.tpmd_destroy.argtypes = [v]
    L.tpmd_last_error.argtypes = [v]
    L.tpmd_last_error.restype = cp
    L.tpmd_scale_for.argtypes = [cp, v]
    L.tpmd_scale_for.restype = C.c_double
    L.tpmd_set_tensor.argtypes = [v, cp, v, i64]
    L.tpmd_prepare.argtypes = [v]
    L.tpmd_set_feats.argtypes = [v, C.POINTER(v)]
    L.tpmd_batch.argtypes = [v]
    L.tpmd_decode.argtypes = [v, v, i64, v]
    L.tpmd_decode_device.argtypes = [v, v, i64, v, v]
    L.tpmd_arena.argtypes = [v, C.c_int, C.POINTER(v), C.POINTER(C.c_size_t)]
    L.tpmd_arena_adopt.argtypes = [v, C.c_int]
    L.tpmd_decode_taps.argtypes = [v, v, C.c_int, v, v, v, v, v]
    L.tpmd_profile_begin.argtypes = [v]
    L.tpmd_profile_end.argtypes = [v, C.c_char_p, C.c_size_t]
    L.tpmd_kernel_launches.argtypes = [v, i64]
    L.tpmd_decode_noalloc.argtypes = [v, v, i64, v, v]
    L.tpmd_device_status.argtypes = [v, v]
    L.tpmd_group_create.argtypes = [C.POINTER(C.c_int), C.c_int, C.c_int, C.c_int]
    L.tpmd_group_create.restype = v
    L.tpmd_group_unique_id.argtypes = [v, C.c_size_t]
    L.tpmd_group_create_rank.argtypes = [C.c_int, C.c_int, C.c_int, v, C.c_size_t, C.c_int, C.c_int]
    L.tpmd_group_create_rank.restype = v
    L.tpmd_group_create_error.restype = cp
    L.tpmd_group_destroy.argtypes = [v]
    L.tpmd_group_last_error.argtypes = [v]
    L.tpmd_group_last_error.restype = cp
    L.tpmd_group_size.argtypes = [v]
    L.tpmd_group_ranks.argtypes = [v, C.POINTER(C.c_int), C.POINTER(C.c_int)]
    L.tpmd_group_member.argtypes = [v, C.c_int]
    L.tpmd_group_member.restype = v
    L.tpmd_group_set_tensor.argtypes = [v, cp, v, i64]
    L.tpmd_group_load_gguf.argtypes = [v, cp]
    L.tpmd_group_prepare.argtypes = [v]
    L.tpmd_group_set_feats.argtypes = [v, C.POINTER(v)]
    L.tpmd_group_set_feats_device.argtypes = [v, C.POINTER(v), v]
    L.tpmd_shard_range.argtypes = [i64, C.c_int, C.c_int, C.POINTER(i64), C.POINTER(i64)]
    L.tpmd_decode_schedule.argtypes = [i64, i64, C.c_int, C.POINTER(i64), i64]
    L.tpmd_decode_schedule.restype = i64
    L.tpmd_group_decode.argtypes = [v, v, i64, v]
    L.tpmd_group_max.argtypes = [v, C.c_double, C.POINTER(C.c_double)]
    L.tpmd_decode_rgb24.argtypes = [v, v, i64, v]
    L.tpmd_group_decode_rgb24.argtypes = [v, v, i64, v]
    L.tpk_chw_to_rgb24.argtypes = [v, i64, C.c_int, C.c_int, v, v]
    L.tpk_gemm.argtypes = [v, i64, v, i64, v, i64, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                           C.c_int, C.c_int, i64, C.c_int, v, C.c_float, C.c_int, v]
    L.tpmd_group_selftest_nccl.argtypes = [C.c_int, C.c_int, C.c_double, C.POINTER(C.c_int), C.c_char_p,
                                           C.c_size_t]
    L.tpmd_debug_expire_wait.argtypes = [v, C.c_longlong]
    L.tpmd_kernel_launches.restype = i64
    L.tpmd_gguf_read.argtypes = [cp, cp, C.c_int, GGUF_TENSOR_FN, v, C.c_char_p, C.c_size_t]
    L.tpmd_load_gguf.argtypes = [v, cp]
    L.tpmd_set_feats_device.argtypes = [v, C.POINTER(v), v]
    L.tpme_create.argtypes = [C.c_int]
    L.tpme_create.restype = v
    L.tpme_create_error.restype = cp
    L.tpme_destroy.argtypes = [v]
    L.tpme_last_error.argtypes = [v]
    L.tpme_last_error.restype = cp
    L.tpme_set_tensor.argtypes = [v, cp, v, i64]
    L.tpme_load_gguf.argtypes = [v, cp]
    L.tpme_prepare.argtypes = [v]
    L.tpme_run.argtypes = [v, v, v, v, v, C.POINTER(v)]
    L.tpme_feat_device.argtypes = [v, C.c_int, C.POINTER(v), C.POINTER(i64)]
    L.tpmd_gguf_read_kv.argtypes = [cp, cp, GGUF_KV_FN, v, C.c_char_p, C.c_size_t]
    L.tpfm_default_config.argtypes = [C.POINTER(FmtConfig)]
    L.tpfm_create.argtypes = [C.c_int, C.c_int, C.POINTER(FmtConfig)]
    L.tpfm_create.restype = v
    L.tpfm_create_error.restype = cp
    L.tpfm_destroy.argtypes = [v]
    L.tpfm_last_error.argtypes = [v]
    L.tpfm_last_error.restype = cp
    L.tpfm_set_tensor.argtypes = [v, cp, v, i64]
    L.tpfm_load_gguf.argtypes = [v, cp]
    L.tpfm_prepare.argtypes = [v]
    L.tpfm_forward.argtypes = [v, v, v, C.c_float, v]
    L.tpfm_sample_chunk.argtypes = [v, v, v, v, v, v, C.c_int, v]
    L.tpae_default_config.argtypes = [C.POINTER(AudConfig)]
    L.tpae_create.argtypes = [C.c_int, C.POINTER(AudConfig)]
    L.tpae_create.restype = v
    L.tpae_create_error.restype = cp
    L.tpae_destroy.argtypes = [v]
    L.tpae_last_error.argtypes = [v]
    L.tpae_last_error.restype = cp
    L.tpae_set_tensor.argtypes = [v, cp, v, i64]
    L.tpae_load_gguf.argtypes = [v, cp]
    L.tpae_prepare.argtypes = [v]
    L.tpae_encode.argtypes = [v, v, i64, i64, v]
    L.tppl_create.argtypes = [C.c_int, cp, C.POINTER(FmtConfig), C.POINTER(AudConfig), C.c_int]
    L.tppl_create.restype = v
    L.tppl_create_error.restype = cp
    L.tppl_destroy.argtypes = [v]
    L.tppl_last_error.argtypes = [v]
    L.tppl_last_error.restype = cp
    L.tppl_load.argtypes = [v, cp]
    for fn in ("tppl_motion_encoder", "tppl_audio_encoder", "tppl_sampler", "tppl_decoder"):
        getattr(L, fn).argtypes = [v]
        getattr(L, fn).restype = v
    L.tppl_prepare.argtypes = [v]
    L.tppl_n_frames.argtypes = [i64]
    L.tppl_n_frames.restype = i64
    L.tppl_n_chunks.argtypes = [i64]
    L.tppl_n_chunks.restype = i64
    L.tppl_generate.argtypes = [v, v, v, i64, C.c_int, v, C.c_uint64, v]
    L.tppl_generate_cb.argtypes = [v, v, v, i64, C.c_int, v, C.c_uint64, FRAME_FN, v]
    L.tppl_styles.argtypes = [v, v, v, i64, C.c_int, v, C.c_uint64, v]
    L.tppl_styles_cb.argtypes = [v, v, v, i64, C.c_int, v, C.c_uint64, STYLES_FN, v]
    L.tpk_bilinear_gather.argtypes = [v, C.c_int, C.c_int, C.c_int, C.c_int, v, i64, C.c_int,
                                      C.c_int, v, v]
    L.tpk_im2col_cf.argtypes = [v] + [C.c_int] * 12 + [v, C.c_int, v]
    L.tpk_last_error.restype = cp
    _lib = L
    return L


GGUF_TENSOR_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_char_p, C.POINTER(C.c_int64),
                             C.POINTER(C.c_float), C.c_int64)


GGUF_KV_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_char_p, C.c_int, C.c_double, C.c_char_p)


class FmtConfig(C.Structure):
    """tpfm_config: the FMT's float.fmt.* hyper-parameters."""
    _fields_ = [(n, C.c_int) for n in ("dim_h", "depth", "n_heads", "dim_w", "dim_a", "dim_e",
                                       "chunk_frames", "prev_frames", "attn_window", "t_freq_dim", "nfe")] + \
               [(n, C.c_float) for n in ("mlp_ratio", "ln_eps", "a_cfg", "e_cfg")]


FRAME_FN = C.CFUNCTYPE(C.c_int, C.c_int64, C.POINTER(C.c_float), C.c_void_p)
STYLES_FN = C.CFUNCTYPE(C.c_int, C.c_int64, C.c_int64, C.POINTER(C.c_float), C.c_void_p)


class AudConfig(C.Structure):
    """tpae_config: the audio encoder's float.audio.* hyper-parameters."""
    _fields_ = [("n_layers", C.c_int), ("n_heads", C.c_int), ("hidden", C.c_int), ("ffn", C.c_int),
                ("dim_w", C.c_int), ("ln_eps", C.c_float), ("conv_dim", C.c_int * 7),
                ("conv_kernel", C.c_int * 7), ("conv_stride", C.c_int * 7), ("pos_kernel", C.c_int),
                ("pos_groups", C.c_int), ("sample_rate", C.c_int), ("fps", C.c_int)]


def _aud_config(cfg: dict) -> AudConfig:
    c = AudConfig()
    for k, val in cfg.items():
        if k.startswith("conv_"):
            getattr(c, k)[:] = list(val)
        else:
            setattr(c, k, val)
    return c


def gguf_kv(path: str, expect_arch: str | None = None) -> dict:
    """The key/value section of a GGUF v3 file through tpmd_gguf_read_kv:
    {key: number or string}."""
    L = load_library()
    out: dict = {}

    def cb(_user, key, vt, num, sv):
        out[key.decode()] = sv.decode() if vt == 8 else num
        return 0

    fn = GGUF_KV_FN(cb)
    err = C.create_string_buffer(1024)
    if L.tpmd_gguf_read_kv(path.encode(), expect_arch.encode() if expect_arch else None, fn, None, err,
                           len(err)) != 0:
        raise TpmdError(err.value.decode())
    return out


def gguf_read(path: str, expect_arch: str | None = None, fold: bool = True) -> dict:
    """Every tensor of a GGUF v3 file as {name: (ne, float32 array)} through
    tpmd_gguf_read (src/gguf_load.cpp:50-197 semantics); ne is the ggml dims
    tuple (fastest first), the array is flat in torch element order, scale
    folded with motion_ae_scale when `fold`."""
    L = load_library()
    out: dict = {}

    def cb(_user, name, ne, data, n):
        out[name.decode()] = (tuple(ne[i] for i in range(4)),
                              np.ctypeslib.as_array(data, shape=(n,)).copy())
        return 0

    fn = GGUF_TENSOR_FN(cb)
    err = C.create_string_buffer(1024)
    rc = L.tpmd_gguf_read(path.encode(), expect_arch.encode() if expect_arch else None,
                          1 if fold else 0, fn, None, err, len(err))
    if rc != 0:
        raise TpmdError(err.value.decode())
    return out


def _np_ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def scale_for(name: str, ne) -> float:
    """motion_ae_scale (src/motion_enc.cpp:14-45) through the C ABI."""
    ne = np.asarray(list(ne) + [1] * (4 - len(ne)), np.int64)
    return load_library().tpmd_scale_for(name.encode(), _np_ptr(ne))


class MotionDecoder:
    """One decoder on one GPU (mirrors the reference's motion_dec:
    prepare / set_feats / decode_batch, src/motion_dec.h:10-49)."""

    def __init__(self, device: int = 0, dtype: int = DTYPE_F16, max_batch: int = 64, _handle=None):
        self._L = load_library()
        self._owned = _handle is None
        self._h = self._L.tpmd_create(device, dtype, max_batch) if _handle is None else _handle
        if not self._h:
            raise TpmdError(self._L.tpmd_create_error().decode())
        self.dtype = dtype
        self.batch = self._L.tpmd_batch(self._h)

    def _check(self, rc: int):
        if rc != 0:
            raise TpmdError(self._L.tpmd_last_error(self._h).decode())

    def set_tensors(self, tensors: dict):
        for name, arr in tensors.items():
            a = np.ascontiguousarray(arr, np.float32)
            self._check(self._L.tpmd_set_tensor(self._h, name.encode(), _np_ptr(a), a.size))

    def load_gguf(self, path: str):
        """The decoder's tensors from a motion_ae GGUF file (tp_ctx::load,
        src/tp.cpp:32-38); call prepare() next."""
        self._check(self._L.tpmd_load_gguf(self._h, path.encode()))

    def prepare(self):
        self._check(self._L.tpmd_prepare(self._h))

    def set_feats_device(self, ptrs, stream: int = 0):
        """The pyramid from device pointers (f32 channel-last), e.g.
        MotionEncoder.feat_ptrs() after a run."""
        arr = (C.c_void_p * N_LEVELS)(*ptrs)
        self._check(self._L.tpmd_set_feats_device(self._h, arr, stream or None))

    def set_feats(self, feats):
        arrs = [np.ascontiguousarray(f, np.float32) for f in feats]
        ptrs = (C.c_void_p * N_LEVELS)(*[a.ctypes.data for a in arrs])
        self._check(self._L.tpmd_set_feats(self._h, ptrs))

    def decode(self, styles: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        """styles [n, 512] f32 (host) -> frames [n, 3, 512, 512] f32 (host)."""
        styles = np.ascontiguousarray(styles, np.float32).reshape(-1, STYLE_DIM)
        n = styles.shape[0]
        if out is None:
            out = np.empty((n, 3, IMG, IMG), np.float32)
        assert out.flags.c_contiguous and out.dtype == np.float32 and out.size == n * 3 * IMG * IMG
        self._check(self._L.tpmd_decode(self._h, _np_ptr(styles), n, _np_ptr(out)))
        return out

    def decode_rgb24(self, styles: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        """styles [n, 512] f32 (host) -> frames [n, 512, 512, 3] uint8 RGB24
        (tpmd_decode_rgb24: converted on the GPU)"""
        styles = np.ascontiguousarray(styles, np.float32).reshape(-1, STYLE_DIM)
        n = styles.shape[0]
        if out is None:
            out = np.empty((n, IMG, IMG, 3), np.uint8)
        assert out.flags.c_contiguous and out.dtype == np.uint8 and out.size == n * 3 * IMG * IMG
        self._check(self._L.tpmd_decode_rgb24(self._h, _np_ptr(styles), n, _np_ptr(out)))
        return out

    def decode_rgb24_ptr(self, styles_ptr: int, n: int, rgb_ptr: int):
        self._check(self._L.tpmd_decode_rgb24(self._h, C.c_void_p(styles_ptr), n, C.c_void_p(rgb_ptr)))

    def decode_ptr(self, styles_ptr: int, n: int, frames_ptr: int):
        """host pointers (e.g. pinned torch tensors' data_ptr())"""
        self._check(self._L.tpmd_decode(self._h, C.c_void_p(styles_ptr), n, C.c_void_p(frames_ptr)))

    def decode_device(self, styles_ptr: int, n: int, frames_ptr: int, stream: int = 0):
        """device pointers, enqueued on `stream` (cudaStream_t as int)"""
        self._check(self._L.tpmd_decode_device(self._h, C.c_void_p(styles_ptr), n,
                                               C.c_void_p(frames_ptr), C.c_void_p(stream)))

    def device_status(self, stream: int = 0):
        """raise TpmdError if a kernel of the device entry points reported an
        expired pipeline wait since the last query (tpmd_device_status)"""
        self._check(self._L.tpmd_device_status(self._h, stream or None))

    def debug_expire_wait(self, wait_ns: int):
        """test hook: the next decode's first tcgen05 conv lets a wait expire"""
        self._check(self._L.tpmd_debug_expire_wait(self._h, int(wait_ns)))

    def taps(self, style: np.ndarray, level: int) -> dict:
        """Parity taps of one frame at `level` (see tpmd_decode_taps)."""
        r, oc = 8 << level, ST_OC[level]
        st = np.ascontiguousarray(style, np.float32).reshape(STYLE_DIM)
        out = {"conv1": np.empty((oc, r, r), np.float32), "conv2": np.empty((oc, r, r), np.float32),
               "rgb": np.empty((3, r, r), np.float32)}
        if level < N_LEVELS - 1:
            out["flowmap"] = np.empty((3, r, r), np.float32)
            out["trunk"] = np.empty((oc, r, r), np.float32)
        p = lambda k: _np_ptr(out[k]) if k in out else None  # noqa: E731
        self._check(self._L.tpmd_decode_taps(self._h, _np_ptr(st), level, p("conv1"), p("conv2"),
                                             p("flowmap"), p("trunk"), p("rgb")))
        return out

    def arena(self, which: int) -> tuple[int, int]:
        p, n = C.c_void_p(), C.c_size_t()
        self._check(self._L.tpmd_arena(self._h, which, C.byref(p), C.byref(n)))
        return p.value, n.value

    def adopt_arena(self, which: int):
        self._check(self._L.tpmd_arena_adopt(self._h, which))

    def profile_begin(self):
        self._check(self._L.tpmd_profile_begin(self._h))

    def profile_end(self) -> dict:
        """{kernel: (launches, total_ms)} timed with CUDA events since begin"""
        import json
        buf = C.create_string_buffer(1 << 16)
        self._check(self._L.tpmd_profile_end(self._h, buf, len(buf)))
        return {k: (v[0], v[1]) for k, v in json.loads(buf.value.decode()).items()}

    def kernel_launches(self, n: int) -> int:
        return self._L.tpmd_kernel_launches(self._h, n)

    def close(self):
        if getattr(self, "_h", None):
            if getattr(self, "_owned", True):
                self._L.tpmd_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()


def _tpk_check(rc: int):
    if rc != 0:
        raise TpmdError(load_library().tpk_last_error().decode())


def bilinear_gather(feat, W: int, H: int, grid, out, planar=False, out_sp=False, stream=0):
    """Device op with ggml_bilinear_gather semantics. feat [W*H, C] (torch CUDA
    f32/f16), grid [N, 2] (or [2, N] planar) f32, out [N, C] (or [C, N])."""
    import torch
    C_ = feat.shape[-1]
    N = grid.numel() // 2
    _tpk_check(load_library().tpk_bilinear_gather(
        C.c_void_p(feat.data_ptr()), int(feat.dtype == torch.float16), C_, W, H,
        C.c_void_p(grid.data_ptr()), N, int(planar), int(out_sp), C.c_void_p(out.data_ptr()),
        C.c_void_p(stream)))
    return out


def chw_to_rgb24(chw, rgb, stream=0):
    """torch CUDA tensors: chw [n, 3, H, W] f32 -> rgb [n, H, W, 3] uint8"""
    n, _, h, w = chw.shape
    _tpk_check(load_library().tpk_chw_to_rgb24(C.c_void_p(chw.data_ptr()), n, h, w,
                                               C.c_void_p(rgb.data_ptr()), C.c_void_p(stream)))


def gemm(X, W, Y, M, N, K, ldx=None, ldw=None, ldy=None, batch=1, x_row_b=0, x_col_b=0, w_row_b=0, w_col_b=0,
         y_batch=0, bias=None, scale=1.0, act=0, stream=0):
    """The library's tcgen05 GEMM on torch CUDA tensors (see tpk_gemm in
    include/tpmd.h): Y = act((X . W^T + bias) * scale), f32 operands by the
    three-pass TF32 split, f16 operands on f16 tensors"""
    import torch
    dt = DTYPE_F16 if X.dtype == torch.float16 else DTYPE_F32
    _tpk_check(load_library().tpk_gemm(
        C.c_void_p(X.data_ptr()), ldx or X.shape[-1], C.c_void_p(W.data_ptr()), ldw or W.shape[-1],
        C.c_void_p(Y.data_ptr()), ldy or Y.shape[-1], M, N, K, batch, x_row_b, x_col_b, w_row_b, w_col_b, y_batch,
        dt, C.c_void_p(bias.data_ptr() if bias is not None else None), scale, act, C.c_void_p(stream)))
    return Y


def im2col_cf(src, IC, IW, IH, N, out, KW=3, KH=3, s0=1, s1=1, p0=1, p1=1, d0=1, d1=1,
              stream=0):
    """Device op with ggml_im2col_cf semantics (see include/tpmd.h)."""
    import torch
    _tpk_check(load_library().tpk_im2col_cf(
        C.c_void_p(src.data_ptr()), IC, IW, IH, N, KW, KH, s0, s1, p0, p1, d0, d1,
        C.c_void_p(out.data_ptr()), int(out.dtype == torch.float16), C.c_void_p(stream)))
    return out


class MotionEncoder:
    """The motion encoder on one GPU (mirrors motion_enc::run,
    src/motion_enc.cpp:46-184): image -> appearance, lambda, motion, feats."""

    def __init__(self, device: int = 0):
        self._L = load_library()
        self._h = self._L.tpme_create(device)
        if not self._h:
            raise TpmdError(self._L.tpme_create_error().decode())

    def _check(self, rc: int):
        if rc != 0:
            raise TpmdError(self._L.tpme_last_error(self._h).decode())

    def set_tensors(self, tensors: dict):
        for name, arr in tensors.items():
            a = np.ascontiguousarray(arr, np.float32)
            self._check(self._L.tpme_set_tensor(self._h, name.encode(), _np_ptr(a), a.size))

    def load_gguf(self, path: str):
        self._check(self._L.tpme_load_gguf(self._h, path.encode()))

    def prepare(self):
        self._check(self._L.tpme_prepare(self._h))

    def run(self, image: np.ndarray, want_feats: bool = True) -> dict:
        img = np.ascontiguousarray(image, np.float32)
        if img.shape != (3, 512, 512):
            raise ValueError("image must be [3, 512, 512] float32 CHW")
        app, lam, mot = np.empty(512, np.float32), np.empty(20, np.float32), np.empty(512, np.float32)
        feats = [np.empty(((8 << j) ** 2, ST_OC[j]), np.float32) for j in range(N_LEVELS)] if want_feats else None
        ptrs = (C.c_void_p * N_LEVELS)(*[f.ctypes.data for f in feats]) if want_feats else None
        self._check(self._L.tpme_run(self._h, _np_ptr(img), _np_ptr(app), _np_ptr(lam), _np_ptr(mot), ptrs))
        return dict(appearance=app, lam=lam, motion=mot, feats=feats)

    def feat_ptrs(self) -> list[int]:
        out = []
        for j in range(N_LEVELS):
            p, n = C.c_void_p(), C.c_int64()
            self._check(self._L.tpme_feat_device(self._h, j, C.byref(p), C.byref(n)))
            out.append(p.value)
        return out

    def close(self):
        if getattr(self, "_h", None):
            self._L.tpme_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class FmtSampler:
    """The flow-matching sampler on one GPU (fmt_model + sample_chunk_ex,
    src/fmt.cpp:9-211, src/pipeline.cpp:15-91)."""

    def __init__(self, cfg: dict, device: int = 0, dtype: int = DTYPE_F32):
        self._L = load_library()
        self.cfg = dict(cfg)
        self._c = FmtConfig(**cfg)
        self._h = self._L.tpfm_create(device, dtype, C.byref(self._c))
        if not self._h:
            raise TpmdError(self._L.tpfm_create_error().decode())

    def _check(self, rc: int):
        if rc != 0:
            raise TpmdError(self._L.tpfm_last_error(self._h).decode())

    def set_tensors(self, tensors: dict):
        for name, arr in tensors.items():
            a = np.ascontiguousarray(arr, np.float32)
            self._check(self._L.tpfm_set_tensor(self._h, name.encode(), _np_ptr(a), a.size))

    def load_gguf(self, path: str):
        self._check(self._L.tpfm_load_gguf(self._h, path.encode()))

    def prepare(self):
        self._check(self._L.tpfm_prepare(self._h))

    def forward(self, x60, cond, t: float) -> np.ndarray:
        c = self.cfg
        T = c["chunk_frames"] + c["prev_frames"]
        x60 = np.ascontiguousarray(x60, np.float32)
        cond = np.ascontiguousarray(cond, np.float32)
        v = np.empty((3, T, c["dim_w"]), np.float32)
        self._check(self._L.tpfm_forward(self._h, _np_ptr(x60), _np_ptr(cond), float(t), _np_ptr(v)))
        return v

    def sample(self, wr, prev_wa, cond_audio, prev_x, x0, emotion: int) -> np.ndarray:
        a = [np.ascontiguousarray(z, np.float32) for z in (wr, prev_wa, cond_audio, prev_x, x0)]
        out = np.empty((self.cfg["chunk_frames"], self.cfg["dim_w"]), np.float32)
        self._check(self._L.tpfm_sample_chunk(self._h, *[_np_ptr(z) for z in a], int(emotion), _np_ptr(out)))
        return out

    def close(self):
        if getattr(self, "_h", None):
            self._L.tpfm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def default_fmt_config() -> dict:
    c = FmtConfig()
    load_library().tpfm_default_config(C.byref(c))
    return {n: getattr(c, n) for n, _ in FmtConfig._fields_}


class AudioEncoder:
    """The audio encoder on one GPU (audio_model::encode,
    src/audio_enc.cpp:55-236): audio -> wa [seq_len, dim_w]."""

    def __init__(self, cfg: dict, device: int = 0):
        self._L = load_library()
        self.cfg = dict(cfg)
        self._c = _aud_config(cfg)
        self._h = self._L.tpae_create(device, C.byref(self._c))
        if not self._h:
            raise TpmdError(self._L.tpae_create_error().decode())

    def _check(self, rc: int):
        if rc != 0:
            raise TpmdError(self._L.tpae_last_error(self._h).decode())

    def set_tensors(self, tensors: dict):
        for name, arr in tensors.items():
            a = np.ascontiguousarray(arr, np.float32)
            self._check(self._L.tpae_set_tensor(self._h, name.encode(), _np_ptr(a), a.size))

    def load_gguf(self, path: str):
        self._check(self._L.tpae_load_gguf(self._h, path.encode()))

    def prepare(self):
        self._check(self._L.tpae_prepare(self._h))

    def encode(self, audio: np.ndarray, seq_len: int) -> np.ndarray:
        a = np.ascontiguousarray(audio, np.float32)
        out = np.empty((seq_len, self.cfg["dim_w"]), np.float32)
        self._check(self._L.tpae_encode(self._h, _np_ptr(a), a.size, seq_len, _np_ptr(out)))
        return out

    def close(self):
        if getattr(self, "_h", None):
            self._L.tpae_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def default_audio_config() -> dict:
    c = AudConfig()
    load_library().tpae_default_config(C.byref(c))
    out = {}
    for n, _ in AudConfig._fields_:
        v = getattr(c, n)
        out[n] = tuple(v) if n.startswith("conv_") else v
    return out


class Pipeline:
    """The end-to-end generator (tppl_*, the reference's generate_impl,
    src/pipeline.cpp:99-186): portrait + audio -> 25 fps frames."""

    def __init__(self, device: int = 0, ftype: str = "f32", fmt_cfg: dict | None = None,
                 audio_cfg: dict | None = None, max_batch: int = 50):
        self._L = load_library()
        fc = C.byref(FmtConfig(**fmt_cfg)) if fmt_cfg else None
        ac = C.byref(_aud_config(audio_cfg)) if audio_cfg else None
        self._h = self._L.tppl_create(device, ftype.encode(), fc, ac, max_batch)
        if not self._h:
            raise TpmdError(self._L.tppl_create_error().decode())

    def _check(self, rc: int):
        if rc < 0:
            raise TpmdError(self._L.tppl_last_error(self._h).decode())
        return rc

    def _set(self, fn_stage, fn_set, tensors):
        h = getattr(self._L, fn_stage)(self._h)
        for name, arr in tensors.items():
            a = np.ascontiguousarray(arr, np.float32)
            if getattr(self._L, fn_set)(h, name.encode(), _np_ptr(a), a.size) != 0:
                raise TpmdError(f"{fn_set}: {name}")

    def set_weights(self, encoder: dict, audio: dict, fmt: dict, decoder: dict):
        self._set("tppl_motion_encoder", "tpme_set_tensor", encoder)
        self._set("tppl_audio_encoder", "tpae_set_tensor", audio)
        self._set("tppl_sampler", "tpfm_set_tensor", fmt)
        self._set("tppl_decoder", "tpmd_set_tensor", decoder)
        self._check(self._L.tppl_prepare(self._h))

    def load(self, gguf_dir: str):
        self._check(self._L.tppl_load(self._h, gguf_dir.encode()))

    def decoder(self) -> "MotionDecoder":
        """The pipeline's own decoder (not owned by the returned object)."""
        return MotionDecoder(0, DTYPE_F16, 1, _handle=self._L.tppl_decoder(self._h))

    def n_frames(self, n_samples: int) -> int:
        return self._L.tppl_n_frames(n_samples)

    def generate(self, image, audio, emotion: int, noise=None, seed: int = 0, out=None) -> np.ndarray:
        img = np.ascontiguousarray(image, np.float32)
        au = np.ascontiguousarray(audio, np.float32)
        n = self.n_frames(au.size)
        if out is None:
            out = np.empty((n, 3, 512, 512), np.float32)
        nz = None if noise is None else np.ascontiguousarray(noise, np.float32)
        self._check(self._L.tppl_generate(self._h, _np_ptr(img), _np_ptr(au), au.size, emotion,
                                          _np_ptr(nz) if nz is not None else None, seed, _np_ptr(out)))
        return out

    def styles(self, image, audio, emotion: int, noise=None, seed: int = 0) -> np.ndarray:
        img = np.ascontiguousarray(image, np.float32)
        au = np.ascontiguousarray(audio, np.float32)
        st = np.empty((self.n_frames(au.size), 512), np.float32)
        nz = None if noise is None else np.ascontiguousarray(noise, np.float32)
        self._check(self._L.tppl_styles(self._h, _np_ptr(img), _np_ptr(au), au.size, emotion,
                                        _np_ptr(nz) if nz is not None else None, seed, _np_ptr(st)))
        return st

    def styles_cb(self, image, audio, emotion: int, cb, noise=None, seed: int = 0) -> int:
        """tppl_styles_cb: cb(frame0, styles [n, 512] view valid during the
        call) after each sampler chunk; a truthy return stops. Returns n_frames."""
        img = np.ascontiguousarray(image, np.float32)
        au = np.ascontiguousarray(audio, np.float32)
        nz = None if noise is None else np.ascontiguousarray(noise, np.float32)
        fn = STYLES_FN(lambda f0, n, p, _u: int(bool(cb(f0, np.ctypeslib.as_array(p, shape=(n, 512))))))
        return self._check(self._L.tppl_styles_cb(self._h, _np_ptr(img), _np_ptr(au), au.size, emotion,
                                                  _np_ptr(nz) if nz is not None else None, seed, fn, None))

    def generate_cb(self, image, audio, emotion: int, cb, noise=None, seed: int = 0) -> int:
        img = np.ascontiguousarray(image, np.float32)
        au = np.ascontiguousarray(audio, np.float32)
        nz = None if noise is None else np.ascontiguousarray(noise, np.float32)
        fn = FRAME_FN(lambda i, p, _u: cb(i, np.ctypeslib.as_array(p, shape=(3, 512, 512))))
        return self._check(self._L.tppl_generate_cb(self._h, _np_ptr(img), _np_ptr(au), au.size, emotion,
                                                    _np_ptr(nz) if nz is not None else None, seed, fn, None))

    def close(self):
        if getattr(self, "_h", None):
            self._L.tppl_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass



def decode_schedule(n: int, max_batch: int, rgb: bool = False) -> list[tuple[int, int, list[int]]]:
    """The host decode's groups (first frame, frames, tail-level part sizes)
    for n >= 4 frames on an f16 handle (tpmd_decode_schedule)"""
    L = load_library()
    cap = 4 * n + 64
    buf = (C.c_int64 * cap)()
    w = L.tpmd_decode_schedule(n, max_batch, 1 if rgb else 0, buf, cap)
    if w < 0:
        raise ValueError("no split schedule for these arguments")
    out, i = [], 0
    while i < w:
        f0, g, k = buf[i], buf[i + 1], buf[i + 2]
        out.append((f0, g, list(buf[i + 3:i + 3 + k])))
        i += 3 + k
    return out


def shard_range(n: int, nranks: int, rank: int) -> tuple[int, int]:
    """[lo, hi) of the frames global rank `rank` decodes (tpmd_shard_range)"""
    L = load_library()
    lo, hi = C.c_int64(), C.c_int64()
    if L.tpmd_shard_range(n, nranks, rank, C.byref(lo), C.byref(hi)) != 0:
        raise ValueError("bad shard arguments")
    return lo.value, hi.value


NCCL_ID_BYTES = 128


def nccl_unique_id() -> bytes:
    """a fresh NCCL clique id for tpmd_group_create_rank (made on rank 0)"""
    L = load_library()
    buf = C.create_string_buffer(NCCL_ID_BYTES)
    if L.tpmd_group_unique_id(buf, NCCL_ID_BYTES) != 0:
        raise TpmdError(L.tpmd_group_create_error().decode())
    return buf.raw


class MotionDecoderGroup:
    """The decoder over several GPUs behind one handle (tpmd_group_*): all of
    `devices` in this process, or (rank, nranks, nccl_id) for one process
    per GPU. Weights and feats are given on global rank 0 and broadcast."""

    def __init__(self, devices=(0,), dtype: int = DTYPE_F16, max_batch: int = 50, rank: int | None = None,
                 nranks: int | None = None, nccl_id: bytes | None = None):
        self._L = load_library()
        if rank is None:
            arr = (C.c_int * len(devices))(*devices)
            self._h = self._L.tpmd_group_create(arr, len(devices), dtype, max_batch)
        else:
            idb = C.create_string_buffer(nccl_id or b"", NCCL_ID_BYTES)
            self._h = self._L.tpmd_group_create_rank(devices[0], rank, nranks, idb, NCCL_ID_BYTES, dtype,
                                                     max_batch)
        if not self._h:
            raise TpmdError(self._L.tpmd_group_create_error().decode())
        r0, nr = C.c_int(), C.c_int()
        self._L.tpmd_group_ranks(self._h, C.byref(r0), C.byref(nr))
        self.rank0, self.nranks = r0.value, nr.value
        self.size = self._L.tpmd_group_size(self._h)
        self.dtype = dtype

    def _check(self, rc: int):
        if rc != 0:
            raise TpmdError(self._L.tpmd_group_last_error(self._h).decode())

    def set_tensors(self, tensors: dict):
        for name, arr in tensors.items():
            a = np.ascontiguousarray(arr, np.float32)
            self._check(self._L.tpmd_group_set_tensor(self._h, name.encode(), _np_ptr(a), a.size))

    def load_gguf(self, path: str):
        self._check(self._L.tpmd_group_load_gguf(self._h, path.encode()))

    def prepare(self):
        self._check(self._L.tpmd_group_prepare(self._h))

    def set_feats(self, feats=None):
        """host feats on global rank 0 (None on the other ranks)"""
        if feats is None:
            feats = [np.zeros(1, np.float32)] * N_LEVELS
        arrs = [np.ascontiguousarray(f, np.float32) for f in feats]
        ptrs = (C.c_void_p * N_LEVELS)(*[a.ctypes.data for a in arrs])
        self._check(self._L.tpmd_group_set_feats(self._h, ptrs))

    def decode(self, styles: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        styles = np.ascontiguousarray(styles, np.float32).reshape(-1, STYLE_DIM)
        n = styles.shape[0]
        if out is None:
            out = np.zeros((n, 3, IMG, IMG), np.float32)
        self._check(self._L.tpmd_group_decode(self._h, _np_ptr(styles), n, _np_ptr(out)))
        return out

    def decode_ptr(self, styles_ptr: int, n: int, frames_ptr: int):
        self._check(self._L.tpmd_group_decode(self._h, C.c_void_p(styles_ptr), n, C.c_void_p(frames_ptr)))

    def decode_rgb24(self, styles: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        styles = np.ascontiguousarray(styles, np.float32).reshape(-1, STYLE_DIM)
        n = styles.shape[0]
        if out is None:
            out = np.zeros((n, IMG, IMG, 3), np.uint8)
        self._check(self._L.tpmd_group_decode_rgb24(self._h, _np_ptr(styles), n, _np_ptr(out)))
        return out

    def member(self, i: int = 0) -> "MotionDecoder":
        """the decoder of local GPU i (not owned: the group frees it)"""
        h = self._L.tpmd_group_member(self._h, i)
        if not h:
            raise TpmdError("no such member")
        return MotionDecoder(_handle=h)

    def max(self, value: float) -> float:
        out = C.c_double()
        self._check(self._L.tpmd_group_max(self._h, float(value), C.byref(out)))
        return out.value

    def close(self):
        if getattr(self, "_h", None):
            self._L.tpmd_group_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()


def nccl_selftest(n: int, scenario: int, limit_s: float) -> tuple[int, int, str]:
    """(rc, aborts, message) of the group's NCCL set-up against a fake NCCL"""
    L = load_library()
    ab = C.c_int()
    err = C.create_string_buffer(256)
    rc = L.tpmd_group_selftest_nccl(n, scenario, limit_s, C.byref(ab), err, len(err))
    return rc, ab.value, err.value.decode()
