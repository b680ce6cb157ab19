"""TEST INFRASTRUCTURE: ctypes wrapper of the C oracle (oracle.c).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs import this module, as
the checker or as the timed CPU baseline. The product path never does.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")


def build() -> str:
    """Compile liboracle.so with oracle/Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(os.path.join(HERE, "oracle.c")):
            build()
        L = C.CDLL(LIB_PATH)
        L.oracle_mat_vec_f16.argtypes = [_u16p, C.c_int64, _f32p, _f32p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        L.oracle_mat_vec_f32.argtypes = [_f32p, _f32p, _f32p] + [C.c_int] * 11 + [C.c_void_p]
        L.oracle_rms_norm.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_float]
        L.oracle_add.argtypes = [_f32p, _f32p, _f32p, C.c_int64]
        L.oracle_swiglu.argtypes = [_f32p, _f32p, _f32p, C.c_int64]
        L.oracle_rope_neox.argtypes = [_f32p, _f32p] + [C.c_int] * 6 + [C.c_float]
        L.oracle_soft_max.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_float]
        L.oracle_argmax.argtypes = [_f32p, C.c_int64]
        L.oracle_argmax.restype = C.c_int
        L.oracle_get_rows_f16.argtypes = [_u16p, C.c_int, C.c_int, _f32p]
        L.oracle_attention.argtypes = [_f32p, _f32p, _f32p, _f32p] + [C.c_int] * 5 + [C.c_float]
        L.oracle_f2h_array.argtypes = [_f32p, _u16p, C.c_int64]
        L.oracle_h2f.argtypes = [C.c_uint16]
        L.oracle_h2f.restype = C.c_float
        L.oracle_qwen2_layer.argtypes = [C.c_void_p, C.c_int, _f32p, C.c_void_p, C.c_void_p, C.c_int, C.c_int]
        L.oracle_qwen2_step.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                        _f32p, C.c_void_p]
        L.oracle_qwen2_step.restype = C.c_int
        L.oracle_mt64_seed.argtypes = [C.c_void_p, C.c_uint64]
        L.oracle_mt64_next.argtypes = [C.c_void_p]
        L.oracle_mt64_next.restype = C.c_uint64
        L.oracle_mt64_bytes.restype = C.c_size_t
        L.oracle_sample.argtypes = [_f32p, C.c_int, C.c_float, C.c_int, C.c_float, C.c_float, C.c_int,
                                    C.c_void_p, C.c_int, C.c_void_p]
        L.oracle_sample.restype = C.c_int
        L.oracle_set_num_threads.argtypes = [C.c_int]
        L.oracle_num_threads.restype = C.c_int
        _lib = L
    return _lib


def set_threads(n: int) -> None:
    lib().oracle_set_num_threads(int(n))


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a) -> int | None:
    return None if a is None else a.ctypes.data


def f16_bits(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float16)).view(np.uint16)


def mat_vec_f16(w16: np.ndarray, x, bias0=None, bias1=None) -> np.ndarray:
    rows, cols = w16.shape
    y = np.empty(rows, np.float32)
    b0 = None if bias0 is None else _f32(bias0)
    b1 = None if bias1 is None else _f32(bias1)
    lib().oracle_mat_vec_f16(f16_bits(w16), cols, _f32(x), y, rows, cols, _ptr(b0), _ptr(b1))
    return y


def mat_vec_f32(a, b, *, ncols, rows, batches, stride_a, batch_stride_a, batch_stride_b, batch_stride_d,
                ne02=1, ne12=1, broadcast2=1, broadcast3=1, bias0=None, d_size=None) -> np.ndarray:
    d = np.zeros(d_size if d_size is not None else batches * batch_stride_d if batches > 1 else rows, np.float32)
    b0 = None if bias0 is None else _f32(bias0)
    lib().oracle_mat_vec_f32(_f32(a), _f32(b), d, ncols, rows, batches, stride_a, batch_stride_a,
                             batch_stride_b, batch_stride_d, ne02, ne12, broadcast2, broadcast3, _ptr(b0))
    return d


def rms_norm(x, w, eps: float) -> np.ndarray:
    x = _f32(x)
    x2 = x.reshape(-1, x.shape[-1])
    y = np.empty_like(x2)
    lib().oracle_rms_norm(x2, _f32(w), y, x2.shape[0], x2.shape[1], eps)
    return y.reshape(x.shape)


def add(a, b) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    d = np.empty_like(a)
    lib().oracle_add(a, b, d, a.size)
    return d


def swiglu(g, u) -> np.ndarray:
    g, u = _f32(g), _f32(u)
    d = np.empty_like(g)
    lib().oracle_swiglu(g, u, d, g.size)
    return d


def rope_neox(x, pos: int, theta_scale: float, n_dims: int | None = None) -> np.ndarray:
    x = _f32(x)
    x2 = x.reshape(-1, x.shape[-1])
    rows, ne00 = x2.shape
    y = np.empty_like(x2)
    lib().oracle_rope_neox(x2, y, rows, ne00, n_dims or ne00, ne00, ne00, pos, theta_scale)
    return y.reshape(x.shape)


def soft_max(x, scale: float) -> np.ndarray:
    x = _f32(x)
    x2 = x.reshape(-1, x.shape[-1])
    y = np.empty_like(x2)
    lib().oracle_soft_max(x2, y, x2.shape[0], x2.shape[1], scale)
    return y.reshape(x.shape)


def argmax(x) -> int:
    x = _f32(x)
    return int(lib().oracle_argmax(x, x.size))


def get_rows_f16(table16: np.ndarray, token: int) -> np.ndarray:
    out = np.empty(table16.shape[1], np.float32)
    lib().oracle_get_rows_f16(f16_bits(table16), table16.shape[1], int(token), out)
    return out


def attention(q, keys, values, heads: int, kv_heads: int, scale: float) -> np.ndarray:
    """q [heads, hd]; keys/values [kv_heads, n, hd] -> [heads, hd]."""
    q, keys, values = _f32(q), _f32(keys), _f32(values)
    kvh, n, hd = keys.shape
    out = np.empty((heads, hd), np.float32)
    lib().oracle_attention(q, keys, values, out, heads, kv_heads, n, hd, n * hd, scale)
    return out


def f2h(x) -> np.ndarray:
    x = _f32(x)
    y = np.empty(x.shape, np.uint16)
    lib().oracle_f2h_array(x.reshape(-1), y.reshape(-1), x.size)
    return y


# ---- Qwen2 model ----------------------------------------------------------------------------------

class _Layer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("attn_norm", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "ffn_norm",
                                           "wgate", "wup", "wdown")]


class _Model(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("layers", "hidden", "ffn", "heads", "kv_heads", "vocab", "max_seq")] + \
               [("eps", C.c_float), ("rope_base", C.c_float), ("token_embd", C.c_void_p), ("output", C.c_void_p),
                ("output_norm", C.c_void_p), ("layer", C.POINTER(_Layer))]


_LAYER_TENSORS = [("attn_norm", "attn_norm.weight"), ("wq", "attn_q.weight"), ("bq", "attn_q.bias"),
                  ("wk", "attn_k.weight"), ("bk", "attn_k.bias"), ("wv", "attn_v.weight"), ("bv", "attn_v.bias"),
                  ("wo", "attn_output.weight"), ("ffn_norm", "ffn_norm.weight"), ("wgate", "ffn_gate.weight"),
                  ("wup", "ffn_up.weight"), ("wdown", "ffn_down.weight")]


class Qwen2:
    """The oracle's view of a synthetic model (``muyo_llm_b200.synth.make_model``), with its caches."""

    def __init__(self, cfg, tensors: dict[str, np.ndarray], kv_f16: bool = False):
        self.cfg = cfg
        self.kv_f16 = kv_f16
        keep = {}
        for k, v in tensors.items():
            keep[k] = np.ascontiguousarray(v.view(np.uint16) if v.dtype == np.float16 else v.astype(np.float32))
        self._keep = keep
        self._layers = (_Layer * cfg.layers)()
        for l in range(cfg.layers):
            for field, suffix in _LAYER_TENSORS:
                setattr(self._layers[l], field, keep[f"blk.{l}.{suffix}"].ctypes.data)
        self._m = _Model(cfg.layers, cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.vocab, cfg.max_seq,
                         cfg.rms_eps, cfg.rope_base, keep["token_embd.weight"].ctypes.data,
                         keep["output.weight"].ctypes.data, keep["output_norm.weight"].ctypes.data, self._layers)
        n = cfg.layers * cfg.kv_heads * cfg.max_seq * cfg.head_dim
        dt = np.uint16 if kv_f16 else np.float32
        self.kcache = np.zeros(n, dt)
        self.vcache = np.zeros(n, dt)

    def reset(self) -> None:
        self.kcache[:] = 0
        self.vcache[:] = 0

    def step(self, token: int, pos: int, want_hidden: bool = False):
        logits = np.empty(self.cfg.vocab, np.float32)
        hidden = np.empty(self.cfg.hidden, np.float32) if want_hidden else None
        arg = lib().oracle_qwen2_step(C.byref(self._m), self.kcache.ctypes.data, self.vcache.ctypes.data,
                                      int(self.kv_f16), int(token), int(pos), logits, _ptr(hidden))
        return (arg, logits, hidden) if want_hidden else (arg, logits)

    def layer(self, l: int, h: np.ndarray, pos: int) -> np.ndarray:
        h = _f32(h).copy()
        cfg = self.cfg
        per = cfg.kv_heads * cfg.max_seq * cfg.head_dim
        lib().oracle_qwen2_layer(C.byref(self._m), l, h, self.kcache[l * per:].ctypes.data,
                                 self.vcache[l * per:].ctypes.data, int(self.kv_f16), int(pos))
        return h


def top2_margin(logits: np.ndarray) -> float:
    top = np.partition(logits, -2)[-2:]
    return float(top[1] - top[0])


def qwen2_greedy(cfg, tensors, forced: list[int], n_total: int, kv_f16: bool = False, threads: int | None = None):
    """Teacher-force ``forced`` then decode greedily up to ``n_total`` ids; returns (ids, margins)
    where margins[i] is the top-1 minus top-2 logit after step i."""
    set_threads(threads or os.cpu_count() or 1)
    m = Qwen2(cfg, tensors, kv_f16=kv_f16)
    seq = list(forced)
    margins = []
    for step in range(n_total - 1):
        arg, logits = m.step(seq[step], step)
        margins.append(top2_margin(logits))
        if step + 1 >= len(seq):
            seq.append(arg)
    return seq, margins


class Sampler:
    """Restatement of the reference's Sampler (src/Sampler.cpp, oracle.c's oracle_sample) with its own
    mt19937_64 state. sample() modifies `logits` in place, as the reference does."""

    def __init__(self, temperature=0.0, top_k=40, top_p=0.95, repeat_penalty=1.0, repeat_last_n=64, seed=0):
        self.params = (float(temperature), int(top_k), float(top_p), float(repeat_penalty), int(repeat_last_n))
        self.state = C.create_string_buffer(int(lib().oracle_mt64_bytes()))
        lib().oracle_mt64_seed(self.state, int(seed))

    def sample(self, logits: np.ndarray, history) -> int:
        assert logits.dtype == np.float32 and logits.flags["C_CONTIGUOUS"]
        h = np.ascontiguousarray(history, dtype=np.int32)
        t, k, p, rp, n = self.params
        return int(lib().oracle_sample(logits, logits.size, t, k, p, rp, n, h.ctypes.data if h.size else None,
                                       h.size, self.state))


REF_SAMPLER = os.path.join(HERE, "_ref", "libsampler_ref.so")


REF_TOKENIZER = os.path.join(HERE, "_ref", "libtokenizer_ref.so")


def reference_tree() -> str | None:
    """The muyo-llm source tree named by the environment variable MUYO_REFERENCE, else by the
    "reference_path" of the repository's BASELINE.json; None unless its sources are there."""
    ref = os.environ.get("MUYO_REFERENCE")
    if not ref:
        try:
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                ref = json.load(f).get("reference_path")
        except (OSError, ValueError):
            ref = None
    return ref if ref and os.path.exists(os.path.join(ref, "src", "Sampler.cpp")) else None


def build_ref() -> str | None:
    """Compile the reference's own sampler and tokenizer into oracle/_ref (needs the reference tree,
    MUYO_REFERENCE); returns the sampler's path, None if neither the tree nor a built copy is there."""
    ref = reference_tree()
    if ref is None:
        return REF_SAMPLER if os.path.exists(REF_SAMPLER) else None
    subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref}"], check=True)
    return REF_SAMPLER


class RefSampler:
    """The reference's Sampler itself (oracle/_ref/libsampler_ref.so, built from src/Sampler.cpp)."""

    def __init__(self, temperature=0.0, top_k=40, top_p=0.95, repeat_penalty=1.0, repeat_last_n=64, seed=0):
        L = C.CDLL(REF_SAMPLER)
        L.ref_sampler_create.argtypes = [C.c_float, C.c_int, C.c_float, C.c_float, C.c_int, C.c_ulonglong]
        L.ref_sampler_create.restype = C.c_void_p
        L.ref_sampler_sample.argtypes = [C.c_void_p, _f32p, C.c_int, C.c_void_p, C.c_int]
        L.ref_sampler_sample.restype = C.c_int
        L.ref_sampler_destroy.argtypes = [C.c_void_p]
        self.L = L
        self.h = L.ref_sampler_create(temperature, top_k, top_p, repeat_penalty, repeat_last_n, seed)

    def sample(self, logits: np.ndarray, history) -> int:
        h = np.ascontiguousarray(history, dtype=np.int32)
        return int(self.L.ref_sampler_sample(self.h, logits, logits.size, h.ctypes.data if h.size else None, h.size))

    def __del__(self):
        try:
            self.L.ref_sampler_destroy(self.h)
        except Exception:
            pass


class RefTokenizer:
    """The reference's Tokenizer itself (oracle/_ref/libtokenizer_ref.so, built from src/Tokenizer.cpp,
    src/Gguf.cpp and the vendored llama.cpp unicode code) over a GGUF file."""

    def __init__(self, path: str):
        L = C.CDLL(REF_TOKENIZER)
        L.ref_tok_open.restype = C.c_void_p
        L.ref_tok_open.argtypes = [C.c_char_p]
        L.ref_tok_close.argtypes = [C.c_void_p]
        L.ref_tok_encode.restype = C.c_long
        L.ref_tok_encode.argtypes = [C.c_void_p, C.c_char_p, C.c_long, C.c_int, C.POINTER(C.c_int), C.c_long]
        L.ref_tok_decode.restype = C.c_long
        L.ref_tok_decode.argtypes = [C.c_void_p, C.POINTER(C.c_int), C.c_long, C.c_char_p, C.c_long]
        L.ref_unicode_flags.argtypes = [C.c_uint, C.c_uint, C.POINTER(C.c_ushort)]
        self.L = L
        self.h = L.ref_tok_open(path.encode())
        if not self.h:
            raise RuntimeError(f"reference tokenizer could not open {path}")

    def encode(self, text: bytes, parse_special: bool = True) -> list[int]:
        buf = (C.c_int * (4 * len(text) + 8))()
        n = self.L.ref_tok_encode(self.h, text, len(text), int(parse_special), buf, len(buf))
        return list(buf[:n])

    def decode(self, ids) -> bytes:
        arr = (C.c_int * max(1, len(ids)))(*ids)
        cap = 64 * len(ids) + 16
        out = C.create_string_buffer(cap)
        n = self.L.ref_tok_decode(self.h, arr, len(ids), out, cap)
        return out.raw[:n]

    @staticmethod
    def unicode_flags() -> np.ndarray:
        """llama.cpp's 16-bit flags of every code point (0x4 letter, 0x2 number, 0x100 white space)."""
        L = C.CDLL(REF_TOKENIZER)
        L.ref_unicode_flags.argtypes = [C.c_uint, C.c_uint, C.POINTER(C.c_ushort)]
        f = np.zeros(0x110000, np.uint16)
        L.ref_unicode_flags(0, f.size, f.ctypes.data_as(C.POINTER(C.c_ushort)))
        return f

    def __del__(self):
        try:
            self.L.ref_tok_close(self.h)
        except Exception:
            pass
