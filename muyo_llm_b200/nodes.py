"""Host-side mirror of the reference's op-node builders: each ``*_params`` function fills the
parameter block exactly as the named node lambda in src/FullModel.cpp fills its push constants,
and each op function calls the matching C-ABI entry point with device buffers (anything with
``data_ptr()``, or a raw int address) on a stream (``None`` = legacy default stream).
"""
from __future__ import annotations

import math

from . import _abi


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t if isinstance(t, int) else t.data_ptr()


def _stream(s):
    if s is None:
        return None
    return s if isinstance(s, int) else s.cuda_stream


# ---- parameter blocks (one per node builder) ------------------------------------------------------

def mat_vec_params(ncols: int, rows: int, *, stride_a: int = 0, stride_b: int = 0, stride_d: int = 0,
                   batch_stride_a: int = 0, batch_stride_b: int = 0, batch_stride_d: int = 0,
                   fusion_flags: int = 0, ne02: int = 1, ne12: int = 1, broadcast2: int = 1, broadcast3: int = 1,
                   batches: int = 1) -> _abi.MatVecParams:
    """MatVecSpec + MatVecExecute (src/FullModel.cpp:133-175): strideD is the row bound."""
    return _abi.MatVecParams(ncols, stride_a or ncols, stride_b or ncols, stride_d or rows, batch_stride_a,
                             batch_stride_b, batch_stride_d, fusion_flags, ne02, ne12, broadcast2, broadcast3, rows,
                             batches)


def _vec4(ne0, ne1=1, ne2=1, ne3=1):
    return ne0, ne1, ne2, ne3, 1, ne0, ne0 * ne1, ne0 * ne1 * ne2


def rms_norm_params(length: int, eps: float, rows: int = 1) -> _abi.BinaryParams:
    """RmsNormExecute (src/FullModel.cpp:215-247), generalised to `rows` rows (src/RmsNorm.cpp)."""
    a = _vec4(length, rows)
    return _abi.BinaryParams(length * rows, *a, length, 1, 1, 1, 1, 0, 0, 0, *a, eps, 0.0, 0)


def add_params(length: int) -> _abi.BinaryParams:
    """AddExecute (src/FullModel.cpp:250-284): two equal-length F32 operands."""
    v = _vec4(length)
    return _abi.BinaryParams(length, *v, *v, *v, 0.0, 0.0, 0)


def get_rows_params(embed_dim: int, vocab: int, n_ids: int = 1) -> _abi.BinaryParams:
    """GetRowsExecute (src/FullModel.cpp:424-458): rows of a [vocab][embed_dim] table."""
    return _abi.BinaryParams(embed_dim * n_ids, embed_dim, vocab, 1, 1, 1, embed_dim, embed_dim * vocab,
                             embed_dim * vocab, n_ids, 1, 1, 1, 1, n_ids, n_ids, n_ids,
                             embed_dim, n_ids, 1, 1, 1, embed_dim, embed_dim * n_ids, embed_dim * n_ids, 0.0, 0.0, 0)


def swiglu_params(count: int, rows: int = 1) -> _abi.GluParams:
    """SwigluExecute (src/FullModel.cpp:287-327): split mode, separate gate and up."""
    n = count * rows
    return _abi.GluParams(n, count, count, _abi.GLU_SPLIT, 0.0, 0.0, 1, count, n, n, 1, count, n, n, 1, count, n, n,
                          rows, 1)


def rope_params(rows: int, head_dim: int, *, input_row_stride: int = 0, output_row_stride: int = 0,
                destination_offset: int = 0, freq_base: float = 10000.0, n_dims: int = 0) -> _abi.RopeParams:
    """RopeSpec + RopeExecute (src/FullModel.cpp:179-212): NEOX, thetaScale = base^(-2/nDims) in float."""
    import numpy as np

    nd = n_dims or head_dim
    theta_scale = float(np.float32(np.power(np.float32(freq_base), np.float32(-2.0) / np.float32(nd))))
    p = _abi.RopeParams()
    p.rope_mode = _abi.ROPE_NEOX
    p.nrows = rows
    p.n_dims = nd
    p.n_offs = 0
    p.freq_scale = 1.0
    p.freq_base = freq_base
    p.attn_factor = 1.0
    p.theta_scale = theta_scale
    p.ne00 = head_dim
    p.ne01 = rows
    p.ne02 = 1
    p.nb01 = input_row_stride or head_dim
    p.nb11 = output_row_stride or head_dim
    p.d_offset = destination_offset
    return p


def soft_max_params(rows: int, columns: int, scale: float) -> _abi.SoftMaxParams:
    """SoftMaxExecute (src/FullModel.cpp:331-349): no mask, scale applied inside."""
    return _abi.SoftMaxParams(columns, 0, columns, rows, 1, 1, 1, 0, 0, 0, scale, 0.0, 0.0, 0.0, 0, rows, 0)


def argmax_params(columns: int, rows: int = 1) -> _abi.GenericParams:
    """ArgmaxExecute (src/FullModel.cpp:461-470)."""
    return _abi.GenericParams(columns, rows, 0.0, 0.0, 0.0, 0.0)


def copy_value_column_params(kv_dim: int, head_dim: int, max_seq: int, position: int) -> _abi.UnaryParams:
    """CopyValueColumnExecute (src/FullModel.cpp:376-420): v[kvh][d] -> vcache[kvh][d][position]."""
    return _abi.UnaryParams(kv_dim, kv_dim, 1, 1, 1, 1, kv_dim, kv_dim, kv_dim,
                            head_dim, max_seq, 1, 1, max_seq, head_dim * max_seq, 0, 0, 0, position)


def attention_params(heads: int, kv_heads: int, head_dim: int, max_seq: int, n_keys: int = 0,
                     kv_dtype: int = _abi.KV_F16, scale: float | None = None) -> _abi.AttentionParams:
    return _abi.AttentionParams(heads, kv_heads, head_dim, max_seq, n_keys, kv_dtype,
                                1.0 / math.sqrt(head_dim) if scale is None else scale)


# ---- ops ------------------------------------------------------------------------------------------

def mat_vec_f16(p, a, b, d, fuse0=None, fuse1=None, stream=None):
    return _abi.call("muyo_cuda_mat_vec_f16", p, _ptr(a), _ptr(b), _ptr(d), _ptr(fuse0), _ptr(fuse1), _stream(stream))


def mat_vec_f32(p, a, b, d, fuse0=None, fuse1=None, stream=None):
    return _abi.call("muyo_cuda_mat_vec_f32", p, _ptr(a), _ptr(b), _ptr(d), _ptr(fuse0), _ptr(fuse1), _stream(stream))


def add(p, a, b, d, stream=None):
    return _abi.call("muyo_cuda_add", p, _ptr(a), _ptr(b), _ptr(d), _stream(stream))


def rms_norm(p, a, w, d, stream=None):
    return _abi.call("muyo_cuda_rms_norm", p, _ptr(a), _ptr(w), _ptr(d), _stream(stream))


def get_rows_f16(p, a, ids, d, stream=None):
    return _abi.call("muyo_cuda_get_rows_f16", p, _ptr(a), _ptr(ids), _ptr(d), _stream(stream))


def get_rows_f32(p, a, ids, d, stream=None):
    return _abi.call("muyo_cuda_get_rows_f32", p, _ptr(a), _ptr(ids), _ptr(d), _stream(stream))


def swiglu(p, a, b, d, stream=None):
    return _abi.call("muyo_cuda_swiglu", p, _ptr(a), _ptr(b), _ptr(d), _stream(stream))


def rope(p, x, pos, d, freq_factors=None, stream=None):
    return _abi.call("muyo_cuda_rope", p, _ptr(x), _ptr(pos), _ptr(freq_factors), _ptr(d), _stream(stream))


def soft_max(p, x, d, mask=None, sinks=None, stream=None):
    return _abi.call("muyo_cuda_soft_max", p, _ptr(x), _ptr(mask), _ptr(sinks), _ptr(d), _stream(stream))


def argmax_workspace_size(p) -> int:
    return int(_abi.lib().muyo_cuda_argmax_workspace_size(p))


def argmax(p, a, d, workspace, workspace_bytes: int, stream=None):
    return _abi.call("muyo_cuda_argmax", p, _ptr(a), _ptr(d), _ptr(workspace), workspace_bytes, _stream(stream))


def copy_f32(p, a, d, stream=None):
    return _abi.call("muyo_cuda_copy_f32", p, _ptr(a), _ptr(d), _stream(stream))


def attention_workspace_size(p) -> int:
    return int(_abi.lib().muyo_cuda_attention_workspace_size(p))


def attention_decode(p, q, k_cache, v_cache, out, workspace, workspace_bytes: int, pos=None, stream=None):
    return _abi.call("muyo_cuda_attention_decode", p, _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(pos), _ptr(out),
                     _ptr(workspace), workspace_bytes, _stream(stream))


def kv_append(p, rope_base: float, k, v, k_cache, v_cache, pos, stream=None):
    return _abi.call("muyo_cuda_kv_append", p, rope_base, _ptr(k), _ptr(v), _ptr(k_cache), _ptr(v_cache), _ptr(pos),
                     _stream(stream))
