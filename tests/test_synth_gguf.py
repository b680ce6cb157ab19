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
