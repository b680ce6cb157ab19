"""Parity of the op-level CUDA kernels (through the C-ABI) with the C oracle.

Configs: the reference's own known-answer checks (src/MatVec.cpp, src/ElementwiseAdd.cpp,
src/RmsNorm.cpp, src/Rope.cpp, src/Swiglu.cpp, src/SoftMax.cpp, src/Argmax.cpp, src/GetRows.cpp),
BASELINE config 1 (GEMV 128x256, U[-1,1]) and config 2 (the op suite at Qwen2.5-0.5B decode shapes,
N(0,1) activations), plus edge cases the kernels branch on.

Tolerances: bit-exact for GEMV on integer inputs, add, get_rows and argmax; otherwise the reference's
|a - e| <= tol * (1 + |e|) with tol = 1e-3 (BASELINE's bound), and the tighter per-check tolerances
of the reference where it states them.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import assert_gemv_accurate, assert_rel_close
from muyo_llm_b200 import _abi, nodes, synth

pytestmark = pytest.mark.gpu
SEED = 7


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def f16(a):
    return np.asarray(a, np.float32).astype(np.float16)


def run_mat_vec_f16(w16, x, bias0=None, bias1=None, rows=None):
    rows = rows or w16.shape[0]
    flags = (_abi.MATVEC_BIAS0 if bias0 is not None else 0) | (_abi.MATVEC_BIAS1 if bias1 is not None else 0)
    d = torch.zeros(rows, dtype=torch.float32, device="cuda")
    W = dev(w16)
    b0 = None if bias0 is None else dev(bias0)
    b1 = None if bias1 is None else dev(bias1)
    nodes.mat_vec_f16(nodes.mat_vec_params(w16.shape[1], rows, fusion_flags=flags), W, dev(x), d, b0, b1)
    return host(d)


def test_matvec_reference_integer_pattern_exact(cuda, oracle_mod):
    # src/MatVec.cpp:68-80,202: exact equality.
    w = np.tile(f16((np.arange(256) % 7) - 3), (128, 1))
    x = ((np.arange(256) % 5) - 2).astype(np.float32)
    got = run_mat_vec_f16(w, x)
    assert (got == oracle_mod.mat_vec_f16(w, x)).all()


def test_matvec_config1_uniform(cuda, oracle_mod):
    # 128 x 256, U[-1,1] weights rounded to F16, U[-1,1] input.
    w = f16(synth.uniform_f32(SEED, "c1.w", (128, 256)))
    x = synth.uniform_f32(SEED, "c1.x", (256,))
    got = run_mat_vec_f16(w, x)
    exp = oracle_mod.mat_vec_f16(w, x)
    assert_rel_close(got, exp, 1e-3, "gemv 128x256")
    assert_gemv_accurate(got, w, x, what="gemv 128x256")


@pytest.mark.parametrize("rows,cols", [(1, 8), (7, 250), (896, 896), (128, 896), (4864, 896), (896, 4864),
                                       (151936, 896), (300, 1000), (33, 4103)])
def test_matvec_shapes(cuda, oracle_mod, rows, cols):
    w = f16(synth.uniform_f32(SEED, f"w{rows}x{cols}", (rows, cols)))
    x = synth.uniform_f32(SEED, f"x{cols}", (cols,))
    got = run_mat_vec_f16(w, x)
    assert_rel_close(got, oracle_mod.mat_vec_f16(w, x), 1e-3, f"gemv {rows}x{cols}")
    assert_gemv_accurate(got, w, x, what=f"gemv {rows}x{cols}")


def test_matvec_bias_fusion(cuda, oracle_mod):
    w = f16(synth.uniform_f32(SEED, "wb", (1152, 896)))
    x = synth.normal_f32(SEED, "xb", (896,))
    b0 = synth.normal_f32(SEED, "b0", (1152,))
    b1 = synth.normal_f32(SEED, "b1", (1152,))
    got0 = run_mat_vec_f16(w, x, b0)
    assert_rel_close(got0, oracle_mod.mat_vec_f16(w, x, b0), 1e-3, "bias0")
    assert_gemv_accurate(got0, w, x, b0, "bias0")
    got1 = run_mat_vec_f16(w, x, b0, b1)
    assert_rel_close(got1, oracle_mod.mat_vec_f16(w, x, b0, b1), 1e-3, "bias0+1")
    assert_gemv_accurate(got1, w, x, b0.astype(np.float64) + b1, "bias0+1")


def test_matvec_unaligned_rows_take_scalar_path(cuda, oracle_mod):
    # Row stride not a multiple of 8 halves and an A pointer 2 bytes off 16: the scalar path.
    rows, cols, ld = 65, 131, 133
    full = f16(synth.uniform_f32(SEED, "ua", (rows * ld + 1,)))
    W = dev(full)
    a_ptr = W.data_ptr() + 2
    x = synth.uniform_f32(SEED, "ux", (cols,))
    d = torch.zeros(rows, dtype=torch.float32, device="cuda")
    nodes.mat_vec_f16(nodes.mat_vec_params(cols, rows, stride_a=ld), a_ptr, dev(x), d)
    w2 = full[1:1 + rows * ld].reshape(rows, ld)[:, :cols]
    assert_rel_close(host(d), oracle_mod.mat_vec_f16(np.ascontiguousarray(w2), x), 1e-3, "unaligned")
    assert_gemv_accurate(host(d), w2, x, what="unaligned")


def test_matvec_f32_gqa_broadcast_scores(cuda, oracle_mod):
    # The attention-score GEMV of src/FullModel.cpp:793-812: K cache [kv][S][hd], q [heads][hd],
    # 14 heads over 2 KV heads (ne12 = broadcast2 = 7), rows = keys so far, stride_d = S.
    kv, heads, hd, S, keys = 2, 14, 64, 256, 37
    K = synth.normal_f32(SEED, "kc", (kv, S, hd))
    q = synth.normal_f32(SEED, "q", (heads, hd))
    p = nodes.mat_vec_params(hd, keys, stride_a=hd, stride_b=hd, stride_d=S, batch_stride_a=hd * S,
                             batch_stride_b=hd, batch_stride_d=S, ne02=1, ne12=7, broadcast2=7, broadcast3=1,
                             batches=heads)
    d = torch.full((heads * S,), -1e30, dtype=torch.float32, device="cuda")
    nodes.mat_vec_f32(p, dev(K), dev(q), d)
    exp = oracle_mod.mat_vec_f32(K, q, ncols=hd, rows=keys, batches=heads, stride_a=hd, batch_stride_a=hd * S,
                                 batch_stride_b=hd, batch_stride_d=S, ne02=1, ne12=7, broadcast2=7, broadcast3=1,
                                 d_size=heads * S)
    got = host(d).reshape(heads, S)
    assert_rel_close(got[:, :keys], exp.reshape(heads, S)[:, :keys], 1e-5, "scores")
    assert (got[:, keys:] == np.float32(-1e30)).all(), "rows past the dispatch must stay untouched"


def test_add_exact(cuda):
    i = np.arange(1000, dtype=np.float32)  # src/ElementwiseAdd.cpp:93-99
    for a, b in [(np.float32(0.5) * i, np.float32(1.0) + np.float32(0.25) * i),
                 (synth.normal_f32(SEED, "a896", (896,)), synth.normal_f32(SEED, "b896", (896,))),
                 (synth.normal_f32(SEED, "a997", (997,)), synth.normal_f32(SEED, "b997", (997,)))]:
        d = torch.empty(a.size, dtype=torch.float32, device="cuda")
        nodes.add(nodes.add_params(a.size), dev(a), dev(b), d)
        assert (host(d) == a + b).all()


def test_add_broadcast(cuda):
    a = synth.normal_f32(SEED, "ab", (4, 96))
    b = synth.normal_f32(SEED, "bb", (96,))
    p = nodes.add_params(96 * 4)
    p.ne00, p.ne01, p.nb01, p.nb02, p.nb03 = 96, 4, 96, 384, 384
    p.ne10, p.ne11, p.nb11, p.nb12, p.nb13 = 96, 1, 96, 96, 96
    p.ne20, p.ne21, p.nb21, p.nb22, p.nb23 = 96, 4, 96, 384, 384
    d = torch.empty(384, dtype=torch.float32, device="cuda")
    nodes.add(p, dev(a), dev(b), d)
    assert (host(d).reshape(4, 96) == a + b[None]).all()


@pytest.mark.parametrize("rows,cols,pattern", [(8, 512, "reference"), (1, 896, "normal"), (8, 512, "normal"),
                                               (3, 4096, "normal"), (2, 37, "normal"), (4, 8192, "normal"),
                                               (2, 8196, "normal"), (5, 1000, "normal")])
def test_rms_norm(cuda, oracle_mod, rows, cols, pattern):
    if pattern == "reference":  # src/RmsNorm.cpp:60-72, tol 1e-4
        r, c = np.meshgrid(np.arange(rows), np.arange(cols), indexing="ij")
        x = (((r * cols + c) % 13) - 6).astype(np.float32)
        w = (np.float32(0.5) + np.float32(0.001) * (np.arange(cols) % 11)).astype(np.float32)
    else:
        x = synth.normal_f32(SEED, f"rn{rows}x{cols}", (rows, cols))
        w = synth.normal_f32(SEED, f"rw{cols}", (cols,))
    d = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    nodes.rms_norm(nodes.rms_norm_params(cols, 1e-6, rows), dev(x), dev(w), d)
    assert_rel_close(host(d).reshape(rows, cols), oracle_mod.rms_norm(x, w, 1e-6), 1e-4, "rms_norm")


def test_swiglu(cuda, oracle_mod):
    i = np.arange(600)  # src/Swiglu.cpp:63-67, tol 1e-5
    g = (np.float32(0.01) * ((i % 17) - 8)).astype(np.float32)
    u = (np.float32(0.5) + np.float32(0.01) * (i % 7)).astype(np.float32)
    for gg, uu in [(g, u), (synth.normal_f32(SEED, "g4864", (4864,)), synth.normal_f32(SEED, "u4864", (4864,)))]:
        d = torch.empty(gg.size, dtype=torch.float32, device="cuda")
        nodes.swiglu(nodes.swiglu_params(gg.size), dev(gg), dev(uu), d)
        assert_rel_close(host(d), oracle_mod.swiglu(gg, uu), 1e-5, "swiglu")


def test_rms_norm_strided_rows(cuda, oracle_mod):
    """Rows with a padded stride take the general kernel; the dense fast path must not be chosen."""
    rows, cols, ld = 3, 512, 520
    x = synth.normal_f32(SEED, "rnpad", (rows, ld))
    w = synth.normal_f32(SEED, "rwpad", (cols,))
    p = nodes.rms_norm_params(cols, 1e-6, rows)
    p.nb01, p.nb02, p.nb03 = ld, ld * rows, ld * rows
    d = torch.zeros(rows * cols, dtype=torch.float32, device="cuda")
    nodes.rms_norm(p, dev(x), dev(w), d)
    assert_rel_close(host(d).reshape(rows, cols), oracle_mod.rms_norm(np.ascontiguousarray(x[:, :cols]), w, 1e-6),
                     1e-4, "rms_norm strided")


@pytest.mark.parametrize("rows,count,pad", [(5, 1000, 0), (3, 4864, 0), (3, 1000, 8), (2, 1002, 0)])
def test_swiglu_rows(cuda, oracle_mod, rows, count, pad):
    """Split mode over several rows: dense rows take the flat float4 path, padded or odd rows the general one."""
    ld = count + pad
    g = synth.normal_f32(SEED, f"gr{rows}x{ld}", (rows, ld))
    u = synth.normal_f32(SEED, f"ur{rows}x{ld}", (rows, ld))
    p = nodes.swiglu_params(count, rows=rows)
    p.nb01, p.nb11 = ld, ld
    p.nb02 = p.nb03 = p.nb12 = p.nb13 = ld * rows
    d = torch.empty(rows * count, dtype=torch.float32, device="cuda")
    nodes.swiglu(p, dev(g), dev(u), d)
    exp = oracle_mod.swiglu(np.ascontiguousarray(g[:, :count]), np.ascontiguousarray(u[:, :count]))
    assert_rel_close(host(d).reshape(rows, count), exp, 1e-5, "swiglu rows")


def test_swiglu_halves_modes(cuda, oracle_mod):
    a = synth.normal_f32(SEED, "glu2", (3, 2 * 100))
    for mode, (gi, ui) in [(_abi.GLU_HALVES, (0, 1)), (_abi.GLU_SWAPPED, (1, 0))]:
        p = nodes.swiglu_params(100, rows=3)
        p.mode, p.ne00, p.nb01, p.nb02, p.nb03 = mode, 200, 200, 600, 600
        d = torch.empty(300, dtype=torch.float32, device="cuda")
        nodes.swiglu(p, dev(a), None, d)
        halves = [a[:, :100], a[:, 100:]]
        exp = oracle_mod.swiglu(np.ascontiguousarray(halves[gi]), np.ascontiguousarray(halves[ui]))
        assert_rel_close(host(d).reshape(3, 100), exp, 1e-5, f"glu mode {mode}")


def _rope_gpu(x, pos, base, rows, hd):
    p = nodes.rope_params(rows, hd, freq_base=base)
    d = torch.empty(rows * hd, dtype=torch.float32, device="cuda")
    nodes.rope(p, dev(x), dev(np.array([pos], np.int32)), d)
    return host(d).reshape(rows, hd), p.theta_scale


def test_rope_reference_check(cuda, oracle_mod):
    x = (np.arange(8) - 3).astype(np.float32)[None]  # src/Rope.cpp:41-64, pos 3, base 1e4, tol 1e-5
    got, ts = _rope_gpu(x, 3, 10000.0, 1, 8)
    assert_rel_close(got, oracle_mod.rope_neox(x, 3, ts), 1e-5, "rope")


@pytest.mark.parametrize("pos", [0, 1, 17, 511, 1023, 2047])
def test_rope_config2(cuda, oracle_mod, pos):
    # 14 query heads + 2 key heads of head_dim 64, theta 1e6.
    x = synth.normal_f32(SEED, f"rope{pos}", (16, 64))
    got, ts = _rope_gpu(x, pos, 1e6, 16, 64)
    assert_rel_close(got, oracle_mod.rope_neox(x, pos, ts), 1e-3, f"rope pos {pos}")


def test_rope_destination_offset_writes_cache_row(cuda, oracle_mod):
    # k_rope of src/FullModel.cpp:771-784: 2 KV heads, out row stride hd*S, dOffset = pos*hd.
    hd, S, pos = 64, 32, 5
    k = synth.normal_f32(SEED, "krope", (2, hd))
    p = nodes.rope_params(2, hd, output_row_stride=hd * S, destination_offset=pos * hd, freq_base=1e6)
    cache = torch.zeros(2 * S * hd, dtype=torch.float32, device="cuda")
    nodes.rope(p, dev(k), dev(np.array([pos], np.int32)), cache)
    c = host(cache).reshape(2, S, hd)
    assert_rel_close(c[:, pos], oracle_mod.rope_neox(k, pos, p.theta_scale), 1e-4, "k rope into cache")
    assert (np.delete(c, pos, axis=1) == 0).all()


@pytest.mark.parametrize("rows,cols,scale", [(1, 64, 0.125), (1, 2048, 1.0), (14, 2048, 0.125), (3, 1000, 0.7)])
def test_soft_max(cuda, oracle_mod, rows, cols, scale):
    if cols == 64:
        x = ((np.arange(64) % 9) - 4).astype(np.float32)[None]  # src/SoftMax.cpp:51-55, tol 1e-5
    else:
        x = synth.normal_f32(SEED, f"sm{rows}x{cols}", (rows, cols))
    d = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    nodes.soft_max(nodes.soft_max_params(rows, cols, scale), dev(x), d)
    assert_rel_close(host(d).reshape(rows, cols), oracle_mod.soft_max(x, scale), 1e-5, "soft_max")


def test_soft_max_masked_tail(cuda):
    # The reference's full-width score row with a -1e30 pre-masked tail (src/FullModel.cpp:63-66,640-641).
    x = np.full((2, 2048), -1e30, np.float32)
    x[:, :100] = synth.normal_f32(SEED, "smtail", (2, 100))
    d = torch.empty(x.size, dtype=torch.float32, device="cuda")
    nodes.soft_max(nodes.soft_max_params(2, 2048, 0.125), dev(x), d)
    got = host(d).reshape(2, 2048)
    v = x[:, :100].astype(np.float64) * 0.125
    e = np.exp(v - v.max(axis=1, keepdims=True))
    assert_rel_close(got[:, :100], e / e.sum(axis=1, keepdims=True), 1e-5, "masked softmax")
    assert (got[:, 100:] == 0).all()


def test_soft_max_mask_and_sinks(cuda):
    rows, cols = 4, 300
    x = synth.normal_f32(SEED, "smx", (rows, cols))
    mask = synth.normal_f32(SEED, "smm", (rows, cols))
    sinks = synth.normal_f32(SEED, "sms", (1,))
    p = nodes.soft_max_params(rows, cols, 0.5)
    p.KY, p.nb11, p.nb12, p.nb13, p.has_sinks = rows, cols, 0, 0, 1
    d = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    nodes.soft_max(p, dev(x), d, mask=dev(mask), sinks=dev(sinks))
    v = x.astype(np.float64) * 0.5 + mask
    m = np.maximum(v.max(axis=1, keepdims=True), sinks[0])
    e = np.exp(v - m)
    exp = e / (e.sum(axis=1, keepdims=True) + np.exp(sinks[0] - m))
    assert_rel_close(host(d).reshape(rows, cols), exp, 1e-5, "soft_max mask+sinks")


def _argmax_gpu(x, rows=1):
    p = nodes.argmax_params(x.size // rows, rows)
    ws_bytes = nodes.argmax_workspace_size(p)
    ws = torch.empty(max(ws_bytes, 8), dtype=torch.uint8, device="cuda")
    d = torch.empty(rows, dtype=torch.int32, device="cuda")
    nodes.argmax(p, dev(x), d, ws, ws_bytes)
    return host(d)


def test_argmax_reference_check(cuda):
    x = (-1.0 + np.float32(0.001) * np.arange(32, dtype=np.float32)).astype(np.float32)
    x[21] = 5.0  # src/Argmax.cpp:51-56,146
    assert _argmax_gpu(x)[0] == 21


def test_argmax_config2_vocab(cuda, oracle_mod):
    x = synth.normal_f32(SEED, "logits", (151936,))
    for where in (0, 151935, 77777):
        y = x.copy()
        y[where] = 100.0
        assert _argmax_gpu(y)[0] == where == oracle_mod.argmax(y)


def test_argmax_ties_first_index(cuda, oracle_mod):
    x = np.zeros(151936, np.float32)
    x[[5000, 9000, 151000]] = 2.0  # max spread over different CTAs: the first index wins
    assert _argmax_gpu(x)[0] == 5000 == oracle_mod.argmax(x)
    assert _argmax_gpu(np.zeros(100, np.float32))[0] == 0
    rows = synth.normal_f32(SEED, "argrows", (5, 20000))
    assert list(_argmax_gpu(rows.reshape(-1), rows=5)) == [oracle_mod.argmax(r) for r in rows]


@pytest.mark.parametrize("rows,cols", [(1, 151937), (3, 99), (2, 8193), (4, 8192), (1, 5)])
def test_argmax_scalar_and_vector_paths(cuda, oracle_mod, rows, cols):
    """Row lengths that are not a multiple of 4 take the scalar scan; the others the float4 scan."""
    x = synth.normal_f32(SEED, f"am{rows}x{cols}", (rows, cols))
    x[:, -1] = 7.5  # the last column, on the ragged edge of both scans
    if rows > 1:
        x[1, 0] = 9.0
    got = _argmax_gpu(x.reshape(-1), rows=rows)
    assert list(got) == [oracle_mod.argmax(r) for r in x]


def test_get_rows(cuda, oracle_mod):
    # src/GetRows.cpp:47-56 pattern (F32 table, exact) and config 2 (row of a 151936 x 896 F16 table).
    t = np.arange(1024)[:, None]
    table32 = ((t % 5) - 2 + np.float32(0.001) * np.arange(512)[None]).astype(np.float32)
    d = torch.empty(512, dtype=torch.float32, device="cuda")
    nodes.get_rows_f32(nodes.get_rows_params(512, 1024), dev(table32), dev(np.array([7], np.int32)), d)
    assert (host(d) == table32[7]).all()
    table16 = f16(synth.normal_f32(SEED, "emb", (151936, 896)) * np.float32(0.02))
    for tok in (0, 12345, 151935):
        d = torch.empty(896, dtype=torch.float32, device="cuda")
        nodes.get_rows_f16(nodes.get_rows_params(896, 151936), dev(table16), dev(np.array([tok], np.int32)), d)
        assert (host(d) == oracle_mod.get_rows_f16(table16, tok)).all()


def test_copy_value_column(cuda):
    # The transposing V append of src/FullModel.cpp:376-420: v[kvh][d] -> vcache[kvh][d][pos].
    kv, hd, S, pos = 2, 64, 128, 9
    v = synth.normal_f32(SEED, "vcol", (kv * hd,))
    cache = torch.zeros(kv * hd * S, dtype=torch.float32, device="cuda")
    nodes.copy_f32(nodes.copy_value_column_params(kv * hd, hd, S, pos), dev(v), cache)
    c = host(cache).reshape(kv, hd, S)
    assert (c[:, :, pos] == v.reshape(kv, hd)).all()
    assert (np.delete(c, pos, axis=2) == 0).all()


def test_abi_rejects_bad_arguments(cuda):
    p = nodes.mat_vec_params(64, 8, fusion_flags=_abi.MATVEC_SCALE0)
    buf = torch.zeros(1024, dtype=torch.float32, device="cuda")
    with pytest.raises(_abi.MuyoError) as e:
        nodes.mat_vec_f16(p, buf, buf, buf)
    assert e.value.rc == -5
    p = nodes.argmax_params(100000)
    with pytest.raises(_abi.MuyoError) as e:
        nodes.argmax(p, buf, buf, buf, 0)
    assert e.value.rc == -1 and "workspace" in str(e.value)
