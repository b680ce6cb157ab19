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
    elif isinstance(value, list) and value and all(isinstance(v, int) for v in value):
        f.write(struct.pack("<IIQ", _ARR, _I32, len(value)))  # e.g. tokenizer.ggml.token_type
        f.write(np.asarray(value, dtype="<i4").tobytes())
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


def gpt2_byte_symbols() -> tuple[list[str], dict[int, str]]:
    """GPT-2's byte -> code point map as the 256 one-symbol tokens, in the order byte-level BPE
    vocabularies list them: the bytes that stand for themselves ('!'..'~', 0xA1..0xAC, 0xAE..0xFF),
    then the other 68 bytes as U+0100.. (so token 0 is "!", as in the Qwen2 and GPT-2 vocabularies)."""
    own = [b for b in range(256) if 0x21 <= b <= 0x7E or 0xA1 <= b <= 0xAC or b >= 0xAE]
    rest = [b for b in range(256) if b not in own]
    cp = {b: b for b in own} | {b: 256 + i for i, b in enumerate(rest)}
    return [chr(cp[b]) for b in own + rest], {b: chr(cp[b]) for b in range(256)}


SPECIALS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]


def bpe_tokenizer(vocab: int, corpus: str, pre: str = "qwen2") -> dict:
    """A byte-level BPE vocabulary of exactly ``vocab`` tokens trained on ``corpus``: the 256 byte
    symbols, ``vocab - 259`` merges (most frequent adjacent pair first, words split at spaces with
    the space kept in front) and the three Qwen2 special tokens (CONTROL, token type 3) at the end.
    Returns the tokenizer.ggml.* metadata, with eos = <|im_end|> and bos = <|endoftext|> as in the
    Qwen2.5 files."""
    symbols, enc = gpt2_byte_symbols()
    n_merges = vocab - 256 - len(SPECIALS)
    assert n_merges >= 0, vocab
    words: dict[tuple[str, ...], int] = {}
    for i, w in enumerate(corpus.split(" ")):
        piece = (" " if i else "") + w
        key = tuple(enc[b] for b in piece.encode())
        if key:
            words[key] = words.get(key, 0) + 1
    tokens, merges = list(symbols), []
    while len(merges) < n_merges:
        pairs: dict[tuple[str, str], int] = {}
        for w, c in words.items():
            for a, b in zip(w, w[1:]):
                pairs[(a, b)] = pairs.get((a, b), 0) + c
        if not pairs:
            break
        best = min(pairs, key=lambda p: (-pairs[p], p))
        merges.append(f"{best[0]} {best[1]}")
        tokens.append(best[0] + best[1])
        merged = {}
        for w, c in words.items():
            out, i = [], 0
            while i < len(w):
                if i + 1 < len(w) and (w[i], w[i + 1]) == best:
                    out.append(w[i] + w[i + 1])
                    i += 2
                else:
                    out.append(w[i])
                    i += 1
            merged[tuple(out)] = merged.get(tuple(out), 0) + c
        words = merged
    while len(tokens) < vocab - len(SPECIALS):  # a corpus too small for the merges asked
        tokens.append(f"<unused{len(tokens)}>")
    tokens += SPECIALS
    types = [1] * (vocab - len(SPECIALS)) + [3] * len(SPECIALS)
    return {
        "tokenizer.ggml.model": "gpt2",
        "tokenizer.ggml.pre": pre,
        "tokenizer.ggml.tokens": tokens,
        "tokenizer.ggml.token_type": types,
        "tokenizer.ggml.merges": merges,
        "tokenizer.ggml.bos_token_id": vocab - 3,
        "tokenizer.ggml.eos_token_id": vocab - 1,
    }


def write_synthetic_qwen2(path: str, cfg: Qwen2Config, seed: int, tokenizer: dict | None = None) -> None:
    """Write the seeded random-init model of ``synth.make_model`` as a Qwen2 GGUF; ``tokenizer``
    (tokenizer.ggml.* keys, e.g. from ``bpe_tokenizer``) replaces the placeholder vocabulary."""
    meta = qwen2_metadata(cfg)
    if tokenizer is not None:
        assert len(tokenizer["tokenizer.ggml.tokens"]) == cfg.vocab
        meta.update(tokenizer)
    write_gguf(path, meta, make_model(cfg, seed))


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
