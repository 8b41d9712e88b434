"""Hugging Face checkpoint loading (wginfer_b200/checkpoint.py), on CPU.

A checkpoint with the reference loader's tensor names
(python/wginfer/models/qwen2.py:75-166) is written in the safetensors layout,
sharded, with tensors that must be skipped; loading it must give back every
weight bit for bit under its ModelWeights name."""
import json
import struct

import numpy as np
import pytest
import torch

from tests.golden import cases as CS
from wginfer_b200 import checkpoint as CK
from wginfer_b200.synthetic import LAYER_NAMES, qwen2_weights

HF_LAYER = {v: k for k, v in CK.LAYER_MAP.items()}


def hf_tensors(w, nlayer, with_lm_head=True):
    t = {"model.embed_tokens.weight": w["in_embed"], "model.norm.weight": w["out_norm_w"]}
    if with_lm_head:
        t["lm_head.weight"] = w["out_embed"]
    for n in LAYER_NAMES:
        for l in range(nlayer):
            t[f"model.layers.{l}.{HF_LAYER[n]}"] = w[n][l]
    return t


def hf_config(cfg, **extra):
    c = {"num_hidden_layers": cfg.nlayer, "hidden_size": cfg.hs, "num_attention_heads": cfg.nh,
         "num_key_value_heads": cfg.nkvh, "intermediate_size": cfg.di, "max_position_embeddings": cfg.maxseq,
         "vocab_size": cfg.voc, "rms_norm_eps": cfg.epsilon, "rope_theta": cfg.theta, "eos_token_id": 7}
    c.update(extra)
    return c


def write_checkpoint(d, cfg, w, with_lm_head=True, **extra):
    t = hf_tensors(w, cfg.nlayer, with_lm_head)
    t["model.layers.0.self_attn.rotary_emb.inv_freq"] = torch.ones(cfg.dh // 2)  # skipped
    t["model.layers.99.mlp.up_proj.weight"] = torch.zeros(2, 2, dtype=torch.bfloat16)  # layer out of range
    names = sorted(t)
    half = len(names) // 2
    CK.write_safetensors(d / "model-00001-of-00002.safetensors", {n: t[n] for n in names[:half]},
                         {"format": "pt"})
    CK.write_safetensors(d / "model-00002-of-00002.safetensors", {n: t[n] for n in names[half:]})
    (d / "config.json").write_text(json.dumps(hf_config(cfg, **extra)))


def test_safetensors_roundtrip_dtypes(tmp_path):
    g = torch.Generator().manual_seed(3)
    ts = {"a": torch.randn(3, 5, generator=g).bfloat16(), "b": torch.randn(7, generator=g),
          "c": torch.randn(2, 2, generator=g).half(), "d": torch.arange(6, dtype=torch.int64).reshape(2, 3),
          "e": torch.zeros(0, 4)}
    CK.write_safetensors(tmp_path / "x.safetensors", ts)
    back = CK.read_safetensors(tmp_path / "x.safetensors")
    assert set(back) == set(ts)
    for k, v in ts.items():
        assert back[k].dtype == v.dtype and tuple(back[k].shape) == tuple(v.shape)
        assert torch.equal(back[k].view(torch.uint8) if v.numel() else back[k], v.view(torch.uint8) if v.numel() else v)


def test_safetensors_layout(tmp_path):
    """The container layout itself: u64 header length, JSON header, data."""
    CK.write_safetensors(tmp_path / "x.safetensors", {"w": torch.tensor([1.0, -2.0])})
    raw = (tmp_path / "x.safetensors").read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    hdr = json.loads(raw[8:8 + n])
    assert hdr["w"] == {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}
    assert np.frombuffer(raw[8 + n:], dtype="<f4").tolist() == [1.0, -2.0]


def test_safetensors_rejects_bad_offsets(tmp_path):
    h = json.dumps({"w": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}).encode()
    (tmp_path / "bad.safetensors").write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 8)
    with pytest.raises(ValueError):
        CK.read_safetensors(tmp_path / "bad.safetensors")


def test_config_from_hf_defaults():
    cfg = CK.config_from_hf({"num_hidden_layers": 28, "hidden_size": 1536, "num_attention_heads": 12,
                             "num_key_value_heads": 2, "intermediate_size": 8960, "vocab_size": 151936,
                             "max_position_embeddings": 131072, "eos_token_id": [151643, 151645]}, maxseq=4096)
    assert (cfg.nlayer, cfg.hs, cfg.nh, cfg.nkvh, cfg.dh, cfg.di, cfg.voc) == (28, 1536, 12, 2, 128, 8960, 151936)
    assert cfg.maxseq == 4096 and cfg.end_token == 151643
    assert cfg.epsilon == 1e-6 and cfg.theta == 1000000.0  # the reference loader's defaults (qwen2.py:39-40)
    assert CK.config_from_hf({"hidden_size": 64, "num_attention_heads": 4}).nkvh == 4


def test_map_name():
    assert CK.map_name("model.layers.3.self_attn.k_proj.bias", 4) == ("attn_k_b", 3)
    assert CK.map_name("model.layers.4.self_attn.k_proj.bias", 4) is None
    assert CK.map_name("model.layers.x.mlp.up_proj.weight", 4) is None
    assert CK.map_name("lm_head.weight", 4) == ("out_embed", -1)
    assert CK.map_name("model.layers.0.self_attn.rotary_emb.inv_freq", 4) is None


def test_load_checkpoint_bit_exact(tmp_path):
    cfg = CS.TINY
    w = qwen2_weights(cfg, seed=4)
    write_checkpoint(tmp_path, cfg, w)
    got, loaded, skipped = CK.load_weights(tmp_path, cfg)
    assert loaded == 3 + cfg.nlayer * len(LAYER_NAMES) and skipped == 2
    for n in ("in_embed", "out_embed", "out_norm_w"):
        assert torch.equal(got[n].view(torch.int16), w[n].view(torch.int16))
    for n in LAYER_NAMES:
        for l in range(cfg.nlayer):
            assert torch.equal(got[n][l].view(torch.int16), w[n][l].view(torch.int16)), (n, l)


def test_load_checkpoint_f32_is_rounded_to_bf16(tmp_path):
    cfg = CS.TINY
    w = qwen2_weights(cfg, seed=5)
    t = {k: v.float() for k, v in hf_tensors(w, cfg.nlayer).items()}
    CK.write_safetensors(tmp_path / "model.safetensors", t)
    got, _, _ = CK.load_weights(tmp_path, cfg)
    assert torch.equal(got["attn_q_w"][1].view(torch.int16), w["attn_q_w"][1].view(torch.int16))


def test_tied_embeddings_and_missing_tensors(tmp_path):
    cfg = CS.TINY
    w = qwen2_weights(cfg, seed=6)
    write_checkpoint(tmp_path, cfg, w, with_lm_head=False)
    with pytest.raises(KeyError, match="out_embed"):
        CK.load_weights(tmp_path, cfg)
    got, _, _ = CK.load_weights(tmp_path, cfg, tie_word_embeddings=True)
    assert got["out_embed"] is got["in_embed"]
    with pytest.raises(FileNotFoundError):
        CK.load_weights(tmp_path / "nowhere", cfg)
