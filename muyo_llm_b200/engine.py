"""Qwen2 decode engine over the C-ABI (muyo_model_*): the host-side mirror of the reference's
``RunFullModel`` (src/FullModel.cpp:487-1291) for Python callers, tests and bench.py.

Weights come from a dict of numpy arrays keyed by GGUF tensor name (``synth.make_model``) or from a
GGUF file; the device owns them afterwards. Every decode step is one replay of the model's CUDA
graph; there is no host computation on the path.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _abi
from .synth import Qwen2Config


def config_struct(cfg: Qwen2Config, kv_dtype: int) -> _abi.Qwen2Config:
    return _abi.Qwen2Config(cfg.layers, cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.vocab, cfg.max_seq,
                            cfg.rms_eps, cfg.rope_base, kv_dtype)


class Qwen2Model:
    """A device-resident Qwen2 model with its KV cache (``kv_dtype``: ``_abi.KV_F16`` or ``KV_F32``)."""

    ENGINE_PERSISTENT, ENGINE_GRAPH = 0, 1

    def __init__(self, cfg: Qwen2Config, tensors: dict | None = None, gguf_path: str | None = None,
                 kv_dtype: int = _abi.KV_F16, device: int = 0, engine: int = 1, pdl: bool = True,
                 prefetch: bool = True, smem_weights: bool = True):
        self.cfg = cfg
        self.kv_dtype = kv_dtype
        self._cfg = config_struct(cfg, kv_dtype)
        handle = C.c_void_p()
        _abi.call("muyo_model_create", C.byref(self._cfg), device, C.byref(handle))
        self._m = handle
        try:
            if gguf_path is not None:
                _abi.call("muyo_model_load_gguf", self._m, gguf_path.encode())
            if tensors is not None:
                for name, arr in tensors.items():
                    if name == "output.weight" and arr is tensors.get("token_embd.weight"):
                        continue  # tied LM head: the model reads token_embd.weight
                    a = np.ascontiguousarray(arr)
                    _abi.call("muyo_model_set_tensor", self._m, name.encode(), a.ctypes.data, a.nbytes)
            _abi.call("muyo_model_set_option", self._m, b"engine", engine)
            _abi.call("muyo_model_set_option", self._m, b"pdl", 1 if pdl else 0)
            _abi.call("muyo_model_set_option", self._m, b"prefetch", 1 if prefetch else 0)
            _abi.call("muyo_model_set_option", self._m, b"smem_weights", 1 if smem_weights else 0)
            _abi.call("muyo_model_finalize", self._m, None)
        except Exception:
            self.close()
            raise

    def close(self) -> None:
        if getattr(self, "_m", None):
            _abi.lib().muyo_model_destroy(self._m)
            self._m = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self, stream=None) -> None:
        _abi.call("muyo_model_reset", self._m, stream)

    @property
    def position(self) -> int:
        p = C.c_int32()
        _abi.call("muyo_model_position", self._m, C.byref(p))
        return p.value

    def set_sampler(self, temperature: float = 0.0, top_k: int = 40, top_p: float = 0.95,
                    repeat_penalty: float = 1.0, repeat_last_n: int = 64, seed: int = 0, stream=None) -> None:
        """Sample generated ids on the device (SamplerParams, src/Sampler.h:14-22; same defaults).
        The defaults (temperature 0, no penalty) are the greedy pick. Re-seeds the engine."""
        p = _abi.SamplerParams(temperature, top_k, top_p, repeat_penalty, repeat_last_n, 0, seed)
        _abi.call("muyo_model_set_sampler", self._m, C.byref(p), stream)

    def generate(self, prompt, n_predict: int, stream=None) -> np.ndarray:
        """Feed ``prompt`` (host ids) and return ``n_predict`` generated ids (host): greedy, or drawn by
        the sampler that set_sampler installed. Blocking."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(max(n_predict, 1), np.int32)
        _abi.call("muyo_model_generate", self._m, p.ctypes.data, p.size, n_predict, out.ctypes.data, stream)
        return out[:n_predict]

    def generate_device(self, prompt_ptr: int, n_prompt: int, n_predict: int, out_ptr: int, stream=None) -> None:
        """Device-buffer variant; asynchronous on ``stream``."""
        _abi.call("muyo_model_generate_device", self._m, prompt_ptr, n_prompt, n_predict, out_ptr, stream)

    def step(self, token: int, want_logits: bool = True, stream=None):
        """One decode step at the current position: (greedy id, logits or None)."""
        nxt = C.c_int32()
        logits = np.empty(self.cfg.vocab, np.float32) if want_logits else None
        _abi.call("muyo_model_step", self._m, int(token), None if logits is None else logits.ctypes.data,
                  C.byref(nxt), stream)
        return nxt.value, logits

    def buffer(self, name: str) -> tuple[int, int]:
        ptr, size = C.c_void_p(), C.c_size_t()
        _abi.call("muyo_model_buffer", self._m, name.encode(), C.byref(ptr), C.byref(size))
        return ptr.value or 0, size.value
