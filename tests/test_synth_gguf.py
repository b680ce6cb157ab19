"""CPU checks of the seeded synthetic model and the GGUF writer/reader."""
from __future__ import annotations

import numpy as np

from muyo_llm_b200 import gguf, synth


def test_tensors_are_deterministic_and_independent():
    cfg = synth.QWEN2_TINY
    a = synth.make_tensor(cfg, 5, "blk.1.ffn_up.weight")
    b = synth.make_tensor(cfg, 5, "blk.1.ffn_up.weight")
    c = synth.make_tensor(cfg, 6, "blk.1.ffn_up.weight")
    assert a.dtype == np.float16 and a.shape == (cfg.ffn, cfg.hidden)
    assert (a.view(np.uint16) == b.view(np.uint16)).all()
    assert not (a.view(np.uint16) == c.view(np.uint16)).all()
    m = synth.make_model(cfg, 5)
    assert m["output.weight"] is m["token_embd.weight"]
    assert abs(float(m["blk.0.attn_q.weight"].astype(np.float32).std()) - 0.02) < 0.002
    assert abs(float(m["blk.0.attn_norm.weight"].mean()) - 1.0) < 0.01


def test_prompt_ids_in_range():
    p = synth.prompt_ids(1, 32, 151936)
    assert p.dtype == np.int32 and p.shape == (32,) and p.min() >= 0 and p.max() < 151936
    assert (p == synth.prompt_ids(1, 32, 151936)).all()


def test_gguf_roundtrip(tmp_path):
    cfg = synth.QWEN2_TINY
    path = str(tmp_path / "m.gguf")
    gguf.write_synthetic_qwen2(path, cfg, 9)
    meta, infos, align = gguf.read_gguf(path)
    assert meta["qwen2.block_count"] == cfg.layers
    assert meta["qwen2.attention.head_count_kv"] == cfg.kv_heads
    assert len(meta["tokenizer.ggml.tokens"]) == cfg.vocab
    assert abs(meta["qwen2.rope.freq_base"] - cfg.rope_base) < 1
    model = synth.make_model(cfg, 9)
    raw = np.fromfile(path, np.uint8)
    for name, (ty, shape, off) in infos.items():
        ref = model[name]
        dt = np.float16 if ty == 1 else np.float32
        assert dt == ref.dtype and tuple(shape) == ref.shape, name
        got = raw[off:off + ref.nbytes].view(dt).reshape(shape)
        assert (got.view(np.uint8) == ref.view(np.uint8)).all(), name
    # the tied LM head shares the embedding's bytes
    assert infos["output.weight"][2] == infos["token_embd.weight"][2]


def test_gguf_qwen2_config_reader(tmp_path):
    """muyo_gguf_read_qwen2_config reads the qwen2.* metadata and the token-list length
    (ReadQwen2Config, src/FullModel.cpp:84-105); metadata only, so it runs without a GPU."""
    import ctypes as C

    from muyo_llm_b200 import _abi, build

    build()
    cfg = synth.QWEN2_TINY
    path = str(tmp_path / "tiny.gguf")
    gguf.write_synthetic_qwen2(path, cfg, 3)
    out = _abi.Qwen2Config()
    _abi.call("muyo_gguf_read_qwen2_config", path.encode(), 64, _abi.KV_F16, C.byref(out))
    assert (out.layers, out.hidden, out.ffn, out.heads, out.kv_heads, out.vocab) == \
        (cfg.layers, cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.vocab)
    assert out.max_seq == 64 and out.kv_dtype == _abi.KV_F16
    assert abs(out.rms_eps - cfg.rms_eps) < 1e-12 and out.rope_base == cfg.rope_base
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOPE" + bytes(20))
    rc = _abi.lib().muyo_gguf_read_qwen2_config(str(bad).encode(), 64, 0, C.byref(out))
    assert _abi.ERRORS.get(rc) == "MUYO_EINVAL"
