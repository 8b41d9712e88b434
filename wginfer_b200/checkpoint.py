"""Qwen2 checkpoints in the Hugging Face layout: config.json + *.safetensors.

Mirrors the reference's loader (python/wginfer/models/qwen2.py:17-166): the
meta fields come from config.json with the same keys and defaults
(qwen2.py:26-41), every tensor is cast to bf16, and checkpoint names map to
the ModelWeights names (qwen2.py:75-166); names that do not map are skipped
and counted. Two additions: `maxseq` may be capped (the reference sizes the
KV cache by `max_position_embeddings`, 131072 for some Qwen2 checkpoints),
and a checkpoint without `lm_head.weight` whose config ties the embeddings
(`tie_word_embeddings`) reuses `model.embed_tokens.weight` as the output
embedding.

The safetensors container is parsed here (8-byte little-endian header
length, a JSON header of {name: {dtype, shape, data_offsets}}, then the raw
little-endian data), so no extra package is needed; tensors are memory
mapped and copied once to the device by `wgb_qwen2_set_weight`.
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np
import torch

from .synthetic import Qwen2Config

_DTYPES = {
    "BF16": (np.uint16, torch.bfloat16), "F16": (np.float16, torch.float16), "F32": (np.float32, torch.float32),
    "F64": (np.float64, torch.float64), "I64": (np.int64, torch.int64), "I32": (np.int32, torch.int32),
    "I16": (np.int16, torch.int16), "I8": (np.int8, torch.int8), "U8": (np.uint8, torch.uint8),
    "BOOL": (np.bool_, torch.bool),
}
_CODES = {v[1]: k for k, v in _DTYPES.items()}

# checkpoint suffix of a layer tensor -> ModelWeights name (qwen2.py:122-163)
LAYER_MAP = {
    "input_layernorm.weight": "attn_norm_w",
    "self_attn.q_proj.weight": "attn_q_w", "self_attn.q_proj.bias": "attn_q_b",
    "self_attn.k_proj.weight": "attn_k_w", "self_attn.k_proj.bias": "attn_k_b",
    "self_attn.v_proj.weight": "attn_v_w", "self_attn.v_proj.bias": "attn_v_b",
    "self_attn.o_proj.weight": "attn_o_w",
    "post_attention_layernorm.weight": "mlp_norm_w",
    "mlp.gate_proj.weight": "mlp_gate_w", "mlp.up_proj.weight": "mlp_up_w", "mlp.down_proj.weight": "mlp_down_w",
}
# global tensors (qwen2.py:77-90)
GLOBAL_MAP = {"model.embed_tokens.weight": "in_embed", "lm_head.weight": "out_embed", "model.norm.weight": "out_norm_w"}


def read_safetensors(path) -> dict:
    """All tensors of one .safetensors file as CPU tensors (memory mapped)."""
    path = Path(path)
    with open(path, "rb") as f:
        head = f.read(8)
        if len(head) != 8:
            raise ValueError(f"{path}: truncated safetensors header")
        (n,) = struct.unpack("<Q", head)
        header = json.loads(f.read(n))
    data = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + n)
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        if info["dtype"] not in _DTYPES:
            raise ValueError(f"{path}: tensor {name} has unsupported dtype {info['dtype']}")
        npdt, tdt = _DTYPES[info["dtype"]]
        b, e = info["data_offsets"]
        if not 0 <= b <= e <= data.size:
            raise ValueError(f"{path}: tensor {name} lies outside the file")
        arr = np.frombuffer(data[b:e], dtype=npdt).reshape(info["shape"])
        t = torch.from_numpy(arr.copy()) if npdt is not np.uint16 else torch.from_numpy(arr.view(np.int16).copy())
        out[name] = t.view(tdt) if npdt is np.uint16 else t
    return out


def write_safetensors(path, tensors: dict, metadata: dict | None = None) -> None:
    """Writes CPU tensors in the safetensors layout (used to make test checkpoints)."""
    header, blobs, off = {}, [], 0
    for name, t in tensors.items():
        t = t.detach().cpu().contiguous()
        raw = t.view(torch.int16).numpy().tobytes() if t.dtype == torch.bfloat16 else t.numpy().tobytes()
        header[name] = {"dtype": _CODES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = metadata
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for raw in blobs:
            f.write(raw)


def config_from_hf(config: dict, maxseq: int | None = None) -> Qwen2Config:
    """ModelMeta from a Hugging Face config.json dict (qwen2.py:26-41)."""
    nh = config.get("num_attention_heads", 0)
    hs = config.get("hidden_size", 0)
    dh = config.get("head_dim", hs // nh if nh else 0) or (hs // nh if nh else 0)
    ms = config.get("max_position_embeddings", 32768)
    eos = config.get("eos_token_id", 151643)
    if isinstance(eos, list):
        eos = eos[0] if eos else -1
    return Qwen2Config(
        nlayer=config.get("num_hidden_layers", config.get("num_layers", 0)), hs=hs, nh=nh,
        nkvh=config.get("num_key_value_heads", nh), dh=dh, di=config.get("intermediate_size", 0),
        maxseq=min(ms, maxseq) if maxseq else ms, voc=config.get("vocab_size", 0),
        epsilon=config.get("rms_norm_eps", 1e-6), theta=config.get("rope_theta", 1000000.0), end_token=eos,
        dtype=torch.bfloat16)


def map_name(key: str, nlayer: int):
    """(ModelWeights name, layer) for a checkpoint tensor name, or None to skip
    (qwen2.py:75-166; layer is -1 for the global tensors)."""
    if key in GLOBAL_MAP:
        return GLOBAL_MAP[key], -1
    if not key.startswith("model.layers."):
        return None
    parts = key.split(".")
    if len(parts) < 4:
        return None
    try:
        layer = int(parts[2])
    except ValueError:
        return None
    if not 0 <= layer < nlayer:
        return None
    name = LAYER_MAP.get(".".join(parts[3:]))
    return (name, layer) if name else None


def load_weights(model_dir, cfg: Qwen2Config, tie_word_embeddings: bool = False):
    """Weights dict in the layout `Qwen2.load_weights` takes (bf16 CPU tensors),
    plus (loaded, skipped) counts."""
    files = sorted(Path(model_dir).glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"No safetensors files found in {model_dir}")
    w = {n: [None] * cfg.nlayer for n in LAYER_MAP.values()}
    loaded = skipped = 0
    for f in files:
        for key, t in read_safetensors(f).items():
            m = map_name(key, cfg.nlayer)
            if m is None:
                skipped += 1
                continue
            name, layer = m
            t = t.to(torch.bfloat16).contiguous()
            if layer < 0:
                w[name] = t
            else:
                w[name][layer] = t
            loaded += 1
    if "out_embed" not in w and tie_word_embeddings and "in_embed" in w:
        w["out_embed"] = w["in_embed"]
    missing = [n for n in GLOBAL_MAP.values() if n not in w]
    missing += [f"{n}[{l}]" for n, ts in w.items() if isinstance(ts, list) for l, t in enumerate(ts)
                if t is None and not (n.endswith("_b") and not cfg.qkv_bias)]
    if missing:
        raise KeyError(f"{model_dir}: checkpoint lacks {', '.join(missing[:8])}" + (" ..." if len(missing) > 8 else ""))
    return w, loaded, skipped


def load_qwen2(model_dir, device: int = 0, max_batch: int = 1, maxseq: int | None = None):
    """A Qwen2 model on the B200 backend from a checkpoint directory."""
    from .qwen2 import Qwen2
    model_dir = Path(model_dir)
    cfg_path = model_dir / "config.json"
    if not cfg_path.exists():
        raise FileNotFoundError(f"config.json not found in {model_dir}")
    config = json.loads(cfg_path.read_text(encoding="utf-8"))
    cfg = config_from_hf(config, maxseq)
    w, _, _ = load_weights(model_dir, cfg, bool(config.get("tie_word_embeddings", False)))
    return Qwen2(cfg, w, device=device, max_batch=max_batch)
