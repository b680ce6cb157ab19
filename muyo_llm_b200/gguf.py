"""Minimal GGUF v3 writer and reader for F32/F16 Qwen2 models.

The reader follows the layout the reference's parser walks (``tools/reference_qwen2.py:10-49``,
``src/Gguf.cpp``): magic, version, tensor count, KV count, the KV pairs, the tensor infos
(name, dims with ``ne0`` first, type, offset) and the data section aligned to
``general.alignment`` (default 32). Only F32 (type 0) and F16 (type 1) tensors are written, the
two types the reference loads (``src/Gguf.cpp:337-348``).

Tied tensors: when two names map to the same numpy array object, the writer emits one data blob
and points both tensor infos at it, so the tied LM head costs no extra bytes on disk.
"""
from __future__ import annotations

import struct
from typing import BinaryIO

import numpy as np

from .synth import Qwen2Config, make_model

_U32, _I32, _F32, _STR, _ARR, _U64 = 4, 5, 6, 8, 9, 10
_ALIGN = 32


def _w_str(f: BinaryIO, s: str) -> None:
    b = s.encode()
    f.write(struct.pack("<Q", len(b)))
    f.write(b)


def _w_kv(f: BinaryIO, key: str, value) -> None:
    _w_str(f, key)
    if isinstance(value, str):
        f.write(struct.pack("<I", _STR))
        _w_str(f, value)
    elif isinstance(value, float):
        f.write(struct.pack("<If", _F32, value))
    elif isinstance(value, int):
        f.write(struct.pack("<II", _U32, value))
    elif isinstance(value, list):
        f.write(struct.pack("<IIQ", _ARR, _STR, len(value)))
        for s in value:
            _w_str(f, s)
    else:
        raise TypeError(f"unsupported GGUF value for {key}: {type(value)}")


def qwen2_metadata(cfg: Qwen2Config) -> dict:
    """The KV pairs the reference reads (``tools/reference_qwen2.py:55-65``, ``src/FullModel.cpp:85-105``)."""
    return {
        "general.architecture": "qwen2",
        "general.alignment": _ALIGN,
        "qwen2.block_count": cfg.layers,
        "qwen2.context_length": cfg.max_seq,
        "qwen2.embedding_length": cfg.hidden,
        "qwen2.feed_forward_length": cfg.ffn,
        "qwen2.attention.head_count": cfg.heads,
        "qwen2.attention.head_count_kv": cfg.kv_heads,
        "qwen2.attention.layer_norm_rms_epsilon": float(cfg.rms_eps),
        "qwen2.rope.freq_base": float(cfg.rope_base),
        # The vocabulary size is the token list's length (src/FullModel.cpp:95).
        "tokenizer.ggml.tokens": [f"<t{i}>" for i in range(cfg.vocab)],
    }


def write_gguf(path: str, metadata: dict, tensors: dict[str, np.ndarray]) -> None:
    blobs: dict[int, int] = {}  # id(array) -> data offset
    order: list[np.ndarray] = []
    infos = []
    offset = 0
    for name, arr in tensors.items():
        if arr.dtype not in (np.float32, np.float16):
            raise TypeError(f"{name}: only F32/F16 tensors are supported")
        key = id(arr)
        if key not in blobs:
            blobs[key] = offset
            order.append(arr)
            offset += (arr.nbytes + _ALIGN - 1) // _ALIGN * _ALIGN
        infos.append((name, arr.shape[::-1], 1 if arr.dtype == np.float16 else 0, blobs[key]))
    with open(path, "wb") as f:
        f.write(b"GGUF")
        f.write(struct.pack("<IQQ", 3, len(infos), len(metadata)))
        for k, v in metadata.items():
            _w_kv(f, k, v)
        for name, dims, ty, off in infos:
            _w_str(f, name)
            f.write(struct.pack("<I", len(dims)))
            for d in dims:
                f.write(struct.pack("<Q", d))
            f.write(struct.pack("<IQ", ty, off))
        pad = (-f.tell()) % _ALIGN
        f.write(b"\0" * pad)
        for arr in order:
            b = np.ascontiguousarray(arr).tobytes()
            f.write(b)
            f.write(b"\0" * ((-len(b)) % _ALIGN))


def write_synthetic_qwen2(path: str, cfg: Qwen2Config, seed: int) -> None:
    """Write the seeded random-init model of ``synth.make_model`` as a Qwen2 GGUF."""
    write_gguf(path, qwen2_metadata(cfg), make_model(cfg, seed))


def read_gguf(path: str) -> tuple[dict, dict[str, tuple[int, tuple[int, ...], int]], int]:
    """Parse a GGUF file: (metadata, {name: (type, C-order shape, absolute offset)}, alignment)."""
    with open(path, "rb") as f:
        def u32():
            return struct.unpack("<I", f.read(4))[0]

        def u64():
            return struct.unpack("<Q", f.read(8))[0]

        def s():
            return f.read(u64()).decode("utf-8", "replace")

        sizes = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}

        def val(t):
            if t == _STR:
                return s()
            if t == _ARR:
                et, n = u32(), u64()
                return [val(et) for _ in range(n)]
            raw = f.read(sizes[t])
            fmt = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q",
                   11: "<q", 12: "<d"}[t]
            return struct.unpack(fmt, raw)[0]

        if f.read(4) != b"GGUF":
            raise ValueError(f"{path}: not a GGUF file")
        _ver, nten, nkv = u32(), u64(), u64()
        meta = {}
        for _ in range(nkv):
            k = s()
            meta[k] = val(u32())
        infos = {}
        for _ in range(nten):
            name = s()
            dims = tuple(u64() for _ in range(u32()))
            ty, off = u32(), u64()
            infos[name] = (ty, dims[::-1], off)
        align = int(meta.get("general.alignment", _ALIGN))
        base = (f.tell() + align - 1) // align * align
    return meta, {k: (t, d, base + o) for k, (t, d, o) in infos.items()}, align
