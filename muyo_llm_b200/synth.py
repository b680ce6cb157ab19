"""Seeded synthetic inputs for the decode-step kernel set.

Every tensor is drawn from its own numpy PCG64 stream, keyed by ``(seed, crc32(name))``, so a
tensor can be regenerated on its own, in any order, on any machine with the same numpy: the GPU
box regenerates byte-identical weights from the seed instead of shipping a 1 GB file.

The model is the Qwen2 architecture the reference decodes (``tools/reference_qwen2.py:51-65``,
``src/FullModel.cpp:69-105``), with GGUF tensor names (``src/FullModel.cpp:582-601``):

* F16 matrices and the tied embedding / LM head: N(0, 0.02), rounded to F16 (round to nearest even);
* F32 QKV biases: N(0, 0.02);
* F32 RMSNorm weights: 1 + N(0, 0.02). The GGUF norms are F32, not the F16 weights the
  N(0, 0.02) rule names; centring them on 1 keeps the activations at unit scale through 24 layers.
"""
from __future__ import annotations

import dataclasses
import zlib

import numpy as np


@dataclasses.dataclass(frozen=True)
class Qwen2Config:
    """The shape fields the reference reads from GGUF metadata (``src/FullModel.cpp:69-105``)."""

    layers: int = 24
    hidden: int = 896
    ffn: int = 4864
    heads: int = 14
    kv_heads: int = 2
    vocab: int = 151936
    rms_eps: float = 1e-6
    rope_base: float = 1e6
    max_seq: int = 2048

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim

    @property
    def gqa(self) -> int:
        return self.heads // self.kv_heads


QWEN2_05B = Qwen2Config()
#: A small model of the same architecture for fast oracle and golden-fixture checks.
QWEN2_TINY = Qwen2Config(layers=2, hidden=64, ffn=128, heads=4, kv_heads=2, vocab=320, max_seq=64)

WEIGHT_STD = 0.02


def tensor_manifest(cfg: Qwen2Config) -> list[tuple[str, tuple[int, ...], str]]:
    """(GGUF name, numpy C-order shape, dtype) for every tensor the decode reads.

    Matrices are ``[out, in]`` in C order, i.e. ggml's ``[ne0 = in, ne1 = out]``
    (``tools/reference_qwen2.py:73-79``). ``output.weight`` is tied to ``token_embd.weight``.
    """
    h, f, q, kv, v = cfg.hidden, cfg.ffn, cfg.q_dim, cfg.kv_dim, cfg.vocab
    out = [("token_embd.weight", (v, h), "f16"), ("output_norm.weight", (h,), "f32"),
           ("output.weight", (v, h), "f16")]
    for layer in range(cfg.layers):
        p = f"blk.{layer}."
        out += [
            (p + "attn_norm.weight", (h,), "f32"),
            (p + "attn_q.weight", (q, h), "f16"), (p + "attn_q.bias", (q,), "f32"),
            (p + "attn_k.weight", (kv, h), "f16"), (p + "attn_k.bias", (kv,), "f32"),
            (p + "attn_v.weight", (kv, h), "f16"), (p + "attn_v.bias", (kv,), "f32"),
            (p + "attn_output.weight", (h, q), "f16"),
            (p + "ffn_norm.weight", (h,), "f32"),
            (p + "ffn_gate.weight", (f, h), "f16"), (p + "ffn_up.weight", (f, h), "f16"),
            (p + "ffn_down.weight", (h, f), "f16"),
        ]
    return out


def _rng(seed: int, name: str) -> np.random.Generator:
    return np.random.default_rng([seed, zlib.crc32(name.encode())])


def make_tensor(cfg: Qwen2Config, seed: int, name: str) -> np.ndarray:
    """Regenerate one tensor of the synthetic model (deterministic in ``seed`` and ``name``)."""
    if name == "output.weight":
        name = "token_embd.weight"  # tied LM head
    shape = dict((n, (s, d)) for n, s, d in tensor_manifest(cfg))[name]
    shp, dtype = shape
    n = int(np.prod(shp))
    rng = _rng(seed, name)
    x = rng.standard_normal(n, dtype=np.float32)
    if name.endswith("norm.weight"):
        x = np.float32(1.0) + x * np.float32(WEIGHT_STD)
    else:
        x = x * np.float32(WEIGHT_STD)
    x = x.reshape(shp)
    return x.astype(np.float16) if dtype == "f16" else x


def make_model(cfg: Qwen2Config, seed: int) -> dict[str, np.ndarray]:
    """All tensors of the synthetic model; ``output.weight`` is the same array as the embedding."""
    out: dict[str, np.ndarray] = {}
    for name, _, _ in tensor_manifest(cfg):
        if name == "output.weight":
            continue
        out[name] = make_tensor(cfg, seed, name)
    out["output.weight"] = out["token_embd.weight"]
    return out


def prompt_ids(seed: int, n: int, vocab: int) -> np.ndarray:
    """The seeded uniform random prompt of the full-model config (ids in ``[0, vocab)``)."""
    return np.random.default_rng([seed, 0x70726F6D]).integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)


def normal_f32(seed: int, tag: str, shape) -> np.ndarray:
    """Seeded N(0, 1) F32 activations for the op-suite and layer configs."""
    n = int(np.prod(shape))
    return _rng(seed, tag).standard_normal(n, dtype=np.float32).reshape(shape)


def uniform_f32(seed: int, tag: str, shape, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
    """Seeded U[lo, hi) F32 values (the GEMV configs' weights and input vectors)."""
    n = int(np.prod(shape))
    return _rng(seed, tag).uniform(lo, hi, size=n).astype(np.float32).reshape(shape)
