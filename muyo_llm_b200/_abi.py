"""ctypes binding of libmuyo_cuda.so (include/muyo_cuda.h). Structures mirror the header field for
field; every call is checked and a failing status raises MuyoError with the library's message.

There is no CPU fallback: if the library is missing, lib() raises, and nothing here computes on the
host.
"""
from __future__ import annotations

import ctypes as C
import os

from . import build as _build

U32 = C.c_uint32
F32 = C.c_float
VP = C.c_void_p

MUYO_OK = 0
ERRORS = {-1: "MUYO_EINVAL", -2: "MUYO_ECUDA", -3: "MUYO_ETIMEOUT", -4: "MUYO_ENOMEM", -5: "MUYO_EUNSUPPORTED",
          -6: "MUYO_ESTATE"}
MATVEC_BIAS0, MATVEC_BIAS1, MATVEC_SCALE0, MATVEC_SCALE1 = 1, 2, 4, 8
MATMUL_BIAS, MATMUL_ACCUMULATE, MATMUL_TCGEN05 = 1, 2, 4
GLU_HALVES, GLU_SWAPPED, GLU_SPLIT = 0, 1, 2
ROPE_NORMAL, ROPE_NEOX = 0, 2
KV_F32, KV_F16 = 0, 1


class MuyoError(RuntimeError):
    def __init__(self, rc: int, msg: str):
        super().__init__(f"{ERRORS.get(rc, rc)}: {msg}")
        self.rc = rc


def _fields(spec: str, ctype=U32):
    return [(n.strip(), ctype) for n in spec.split(",") if n.strip()]


class MatVecParams(C.Structure):
    _fields_ = _fields("ncols, stride_a, stride_b, stride_d, batch_stride_a, batch_stride_b, batch_stride_d, "
                       "fusion_flags, ne02, ne12, broadcast2, broadcast3, rows, batches")


class BinaryParams(C.Structure):
    _fields_ = _fields("ne, ne00, ne01, ne02, ne03, nb00, nb01, nb02, nb03, ne10, ne11, ne12, ne13, nb10, nb11, nb12, "
                       "nb13, ne20, ne21, ne22, ne23, nb20, nb21, nb22, nb23") + \
               [("param1", F32), ("param2", F32), ("param3", C.c_int32)]


class GluParams(C.Structure):
    _fields_ = _fields("N, ne00, ne20, mode") + [("alpha", F32), ("limit", F32)] + \
               _fields("nb00, nb01, nb02, nb03, nb10, nb11, nb12, nb13, nb20, nb21, nb22, nb23, ne21, ne22")


class RopeParams(C.Structure):
    _fields_ = _fields("rope_mode, nrows, n_dims, n_offs") + \
               _fields("freq_scale, freq_base, ext_factor, attn_factor", F32) + [("corr_dims", F32 * 2),
                                                                                  ("theta_scale", F32)] + \
               _fields("has_ff, is_back, ne00, ne01, ne02, nb01, nb02, nb03, nb11, nb12, nb13, a_offset, d_offset")


class SoftMaxParams(C.Structure):
    _fields_ = _fields("KX, KY, ne00, ne01, ne02, ne12, ne13, nb11, nb12, nb13") + \
               _fields("scale, max_bias, m0, m1", F32) + _fields("n_head_log2, nrows_x, has_sinks")


class GenericParams(C.Structure):
    _fields_ = _fields("KX, KY") + _fields("param1, param2, param3, param4", F32)


class UnaryParams(C.Structure):
    _fields_ = _fields("ne, ne00, ne01, ne02, ne03, nb00, nb01, nb02, nb03, ne10, ne11, ne12, ne13, nb10, nb11, nb12, "
                       "nb13, a_offset, d_offset")


class AttentionParams(C.Structure):
    _fields_ = _fields("heads, kv_heads, head_dim, max_seq, n_keys, kv_dtype") + [("scale", F32)]


class Qwen2Config(C.Structure):
    _fields_ = _fields("layers, hidden, ffn, heads, kv_heads, vocab, max_seq") + \
               [("rms_eps", F32), ("rope_base", F32), ("kv_dtype", U32)]


class MatMulParams(C.Structure):
    _fields_ = [(n, U32) for n in ("ncols", "rows", "tokens", "stride_x", "stride_y", "flags")]


class SamplerParams(C.Structure):
    _fields_ = [("temperature", F32), ("top_k", C.c_int32), ("top_p", F32), ("repeat_penalty", F32),
                ("repeat_last_n", C.c_int32), ("cluster_ctas", U32), ("seed", C.c_uint64)]


class LayerWeights(C.Structure):
    _fields_ = [(n, VP) for n in ("attn_norm", "wqkv", "bqkv", "wo", "ffn_norm", "wgate", "wup", "wdown")]


P = C.POINTER
# name -> (restype, argtypes)
SIGNATURES = {
    "muyo_cuda_init": (C.c_int, [C.c_int]),
    "muyo_cuda_shutdown": (C.c_int, []),
    "muyo_cuda_last_error": (C.c_char_p, []),
    "muyo_cuda_version": (C.c_char_p, []),
    "muyo_cuda_mat_vec_f16": (C.c_int, [P(MatVecParams), VP, VP, VP, VP, VP, VP]),
    "muyo_cuda_mat_vec_f32": (C.c_int, [P(MatVecParams), VP, VP, VP, VP, VP, VP]),
    "muyo_cuda_add": (C.c_int, [P(BinaryParams), VP, VP, VP, VP]),
    "muyo_cuda_rms_norm": (C.c_int, [P(BinaryParams), VP, VP, VP, VP]),
    "muyo_cuda_get_rows_f16": (C.c_int, [P(BinaryParams), VP, VP, VP, VP]),
    "muyo_cuda_get_rows_f32": (C.c_int, [P(BinaryParams), VP, VP, VP, VP]),
    "muyo_cuda_swiglu": (C.c_int, [P(GluParams), VP, VP, VP, VP]),
    "muyo_cuda_rope": (C.c_int, [P(RopeParams), VP, VP, VP, VP, VP]),
    "muyo_cuda_soft_max": (C.c_int, [P(SoftMaxParams), VP, VP, VP, VP, VP]),
    "muyo_cuda_argmax_workspace_size": (C.c_size_t, [P(GenericParams)]),
    "muyo_cuda_argmax": (C.c_int, [P(GenericParams), VP, VP, VP, C.c_size_t, VP]),
    "muyo_cuda_copy_f32": (C.c_int, [P(UnaryParams), VP, VP, VP]),
    "muyo_cuda_attention_workspace_size": (C.c_size_t, [P(AttentionParams)]),
    "muyo_cuda_attention_decode": (C.c_int, [P(AttentionParams), VP, VP, VP, VP, VP, VP, C.c_size_t, VP]),
    "muyo_cuda_kv_append": (C.c_int, [P(AttentionParams), F32, VP, VP, VP, VP, VP, VP]),
    "muyo_cuda_layer_workspace_size": (C.c_size_t, [P(Qwen2Config)]),
    "muyo_cuda_layer_step": (C.c_int, [P(Qwen2Config), P(LayerWeights), VP, VP, VP, VP, VP, VP, C.c_size_t, VP]),
    "muyo_model_create": (C.c_int, [P(Qwen2Config), C.c_int, P(VP)]),
    "muyo_model_set_tensor": (C.c_int, [VP, C.c_char_p, VP, C.c_size_t]),
    "muyo_model_load_gguf": (C.c_int, [VP, C.c_char_p]),
    "muyo_gguf_read_qwen2_config": (C.c_int, [C.c_char_p, U32, U32, P(Qwen2Config)]),
    "muyo_model_finalize": (C.c_int, [VP, VP]),
    "muyo_model_reset": (C.c_int, [VP, VP]),
    "muyo_model_generate": (C.c_int, [VP, VP, C.c_int, C.c_int, VP, VP]),
    "muyo_model_generate_device": (C.c_int, [VP, VP, C.c_int, C.c_int, VP, VP]),
    "muyo_model_step": (C.c_int, [VP, C.c_int32, VP, VP, VP]),
    "muyo_model_position": (C.c_int, [VP, P(C.c_int32)]),
    "muyo_model_buffer": (C.c_int, [VP, C.c_char_p, P(VP), P(C.c_size_t)]),
    "muyo_model_destroy": (C.c_int, [VP]),
    "muyo_model_set_option": (C.c_int, [VP, C.c_char_p, C.c_int]),
    "muyo_cuda_mat_vec_f16_argmax": (C.c_int, [P(MatVecParams), VP, VP, VP, U32, VP, VP, C.c_size_t, VP]),
    "muyo_cuda_argmax_pairs": (C.c_int, [VP, U32, VP, VP]),
    "muyo_cuda_argmax_noalloc_max_pairs": (C.c_size_t, []),
    "muyo_cuda_argmax_noalloc": (C.c_int, [P(GenericParams), VP, VP, VP]),
    "muyo_sampler_state_bytes": (C.c_size_t, []),
    "muyo_sampler_seed": (C.c_int, [VP, C.c_uint64, VP]),
    "muyo_cuda_sample": (C.c_int, [P(SamplerParams), VP, U32, VP, U32, VP, VP, VP]),
    "muyo_model_set_sampler": (C.c_int, [VP, P(SamplerParams), VP]),
    "muyo_cuda_mat_mul_f16_workspace_size": (C.c_size_t, [P(MatMulParams)]),
    "muyo_cuda_mat_mul_f16": (C.c_int, [P(MatMulParams), VP, VP, VP, VP, VP, C.c_size_t, VP]),
    "muyo_p2p_handle_bytes": (C.c_size_t, []),
    "muyo_p2p_create": (C.c_int, [C.c_int, C.c_int, U32, P(VP), VP]),
    "muyo_p2p_connect": (C.c_int, [VP, VP]),
    "muyo_cuda_mat_vec_f16_allgather": (C.c_int, [VP, P(MatVecParams), VP, VP, U32, VP, VP]),
    "muyo_p2p_output": (C.c_int, [VP, P(VP)]),
    "muyo_p2p_check": (C.c_int, [VP]),
    "muyo_p2p_destroy": (C.c_int, [VP]),
}

_lib = None


def lib_path() -> str:
    return _build.LIB


def lib() -> C.CDLL:
    """Load the in-tree library (built by ``muyo_llm_b200.build``). Raises if it is missing."""
    global _lib
    if _lib is None:
        path = lib_path()
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: run `python -m muyo_llm_b200.build` (no CPU fallback exists)")
        L = C.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return (lib().muyo_cuda_last_error() or b"").decode()


def check(rc: int) -> int:
    if rc != MUYO_OK:
        raise MuyoError(rc, last_error())
    return rc


def call(name: str, *args) -> int:
    """Call an int-returning entry point and raise MuyoError on a failing status."""
    return check(getattr(lib(), name)(*args))
