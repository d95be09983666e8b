"""Minimal GGUF v3 writer for tests: the layout the reference's converter
produces for motion_ae files (verbatim torch names, dims reversed from torch
so ne[0] is the last torch dim, 5-D modconv weights kept 5-D, 32-byte
alignment, general.architecture "float-motion-ae"), written from the GGUF v3
format description. Also able to write malformed files for the reader's
error paths."""
from __future__ import annotations

import re
import struct

import numpy as np

ALIGN = 32
T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARRAY = 4, 5, 6, 7, 8, 9

# modulated convs carry a leading singleton in torch: [1, OC, IC, k, k]
_MODCONV = re.compile(r"^dec\.(conv1|convs\.\d+|to_flows\.\d+)\.conv\.weight$")


def torch_shape(name: str, shape: tuple) -> tuple:
    """The parameter's torch shape as the converter sees it."""
    return (1,) + tuple(shape) if _MODCONV.match(name) else tuple(shape)


def _s(x: str) -> bytes:
    b = x.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vt: int, val) -> bytes:
    out = _s(key) + struct.pack("<I", vt)
    if vt == T_U32:
        return out + struct.pack("<I", val)
    if vt == T_I32:
        return out + struct.pack("<i", val)
    if vt == T_F32:
        return out + struct.pack("<f", val)
    if vt == T_BOOL:
        return out + struct.pack("<B", 1 if val else 0)
    if vt == T_STR:
        return out + _s(val)
    if vt == T_ARRAY:  # array of u32 (not accepted by the reader)
        return out + struct.pack("<IQ", T_U32, len(val)) + b"".join(struct.pack("<I", v) for v in val)
    raise ValueError(vt)


def write(path: str, tensors: list, arch: str | None = "float-motion-ae", extra_kv: list | None = None,
          version: int = 3, magic: bytes = b"GGUF", type_override: dict | None = None,
          offset_override: dict | None = None, truncate: int | None = None) -> None:
    """tensors: [(name, array in torch shape, 'f32' | 'f16')]."""
    kvs = []
    if arch is not None:
        kvs.append(_kv("general.architecture", T_STR, arch))
    kvs.append(_kv("general.alignment", T_U32, ALIGN))
    for k in extra_kv or []:
        kvs.append(_kv(*k))
    infos, blobs, off = [], [], 0
    for name, arr, dt in tensors:
        a = np.ascontiguousarray(arr, np.float16 if dt == "f16" else np.float32)
        ne = list(reversed(a.shape))
        gtype = 1 if dt == "f16" else 0
        if type_override and name in type_override:
            gtype = type_override[name]
        o = offset_override.get(name, off) if offset_override else off
        infos.append(_s(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", d) for d in ne)
                     + struct.pack("<IQ", gtype, o))
        raw = a.tobytes()
        pad = (-len(raw)) % ALIGN
        blobs.append(raw + b"\0" * pad)
        off += len(raw) + pad
    head = magic + struct.pack("<IQQ", version, len(tensors), len(kvs)) + b"".join(kvs) + b"".join(infos)
    head += b"\0" * ((-len(head)) % ALIGN)
    data = head + b"".join(blobs)
    if truncate is not None:
        data = data[:truncate]
    with open(path, "wb") as f:
        f.write(data)
