"""Seeded synthetic inputs and Qwen2 weights (no checkpoints exist offline).

Distributions: activations ~N(0, 1); linear weights, biases and both
embedding tables ~N(0, 0.02); RMSNorm weights ~N(1, 0.1). Values are drawn
in f32 from one ``torch.Generator`` seeded with ``seed`` in a fixed tensor
order, then rounded to the model dtype (round-to-nearest-even), so the same
seed gives the same bits on every machine.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

LAYER_NAMES = ("attn_norm_w", "attn_q_w", "attn_q_b", "attn_k_w", "attn_k_b", "attn_v_w",
               "attn_v_b", "attn_o_w", "mlp_norm_w", "mlp_gate_w", "mlp_up_w", "mlp_down_w")


@dataclass
class Qwen2Config:
    """Mirror of the reference's ModelMeta (src/models/qwen2/model.hpp:18-31)."""
    nlayer: int = 28
    hs: int = 1536
    nh: int = 12
    nkvh: int = 2
    dh: int = 128
    di: int = 8960
    maxseq: int = 1024
    voc: int = 151936
    epsilon: float = 1e-6
    theta: float = 1e4
    end_token: int = -1
    dtype: torch.dtype = torch.bfloat16
    qkv_bias: bool = True

    def shapes(self):
        hs, nh, nkvh, dh, di = self.hs, self.nh, self.nkvh, self.dh, self.di
        return {
            "attn_norm_w": (hs,), "attn_q_w": (nh * dh, hs), "attn_q_b": (nh * dh,),
            "attn_k_w": (nkvh * dh, hs), "attn_k_b": (nkvh * dh,),
            "attn_v_w": (nkvh * dh, hs), "attn_v_b": (nkvh * dh,),
            "attn_o_w": (hs, nh * dh), "mlp_norm_w": (hs,), "mlp_gate_w": (di, hs),
            "mlp_up_w": (di, hs), "mlp_down_w": (hs, di),
        }

    def weight_bytes(self) -> int:
        """Bytes of every weight one batch-1 decode step streams (all linears,
        biases and norms plus lm_head; the embedding gathers one row)."""
        es = torch.tensor([], dtype=self.dtype).element_size()
        per_layer = 0
        for n, s in self.shapes().items():
            if n.endswith("_b") and not self.qkv_bias:
                continue
            k = 1
            for d in s:
                k *= d
            per_layer += k
        return es * (self.nlayer * per_layer + self.voc * self.hs + self.hs)


# Qwen2-1.5B architecture (DeepSeek-R1-Distill-Qwen-1.5B shapes).
QWEN2_1P5B = Qwen2Config()


def _draw(gen, shape, std, mean, dtype, device):
    t = torch.randn(shape, generator=gen, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    if mean != 0.0:
        t.add_(mean)
    return t.to(dtype=dtype).to(device)


def qwen2_weights(cfg: Qwen2Config, seed: int = 0, device="cpu") -> dict:
    """Weights in the fixed order in_embed, per layer LAYER_NAMES, out_norm_w,
    out_embed. Per-layer entries are lists indexed by layer."""
    gen = torch.Generator("cpu").manual_seed(seed)
    w = {"in_embed": _draw(gen, (cfg.voc, cfg.hs), 0.02, 0.0, cfg.dtype, device)}
    for n in LAYER_NAMES:
        w[n] = []
    shapes = cfg.shapes()
    for _ in range(cfg.nlayer):
        for n in LAYER_NAMES:
            if n.endswith("_b") and not cfg.qkv_bias:
                w[n].append(None)
                continue
            if n.endswith("norm_w"):
                w[n].append(_draw(gen, shapes[n], 0.1, 1.0, cfg.dtype, device))
            else:
                w[n].append(_draw(gen, shapes[n], 0.02, 0.0, cfg.dtype, device))
    w["out_norm_w"] = _draw(gen, (cfg.hs,), 0.1, 1.0, cfg.dtype, device)
    w["out_embed"] = _draw(gen, (cfg.voc, cfg.hs), 0.02, 0.0, cfg.dtype, device)
    return w


def prompt_ids(n: int, voc: int, seed: int = 0, batch: int | None = None) -> torch.Tensor:
    """Uniform token ids in [0, voc) from the seed (shape [n] or [batch, n])."""
    gen = torch.Generator("cpu").manual_seed(seed + 7919)
    shape = (n,) if batch is None else (batch, n)
    return torch.randint(0, voc, shape, generator=gen, dtype=torch.int64)


def activations(shape, dtype=torch.float32, seed: int = 0, std: float = 1.0) -> torch.Tensor:
    gen = torch.Generator("cpu").manual_seed(seed)
    return _draw(gen, shape, std, 0.0, dtype, "cpu")


def to_numpy_bits(t: torch.Tensor):
    """Host numpy view of a tensor's bits (bf16/f16 as uint16, f32 as float32)."""
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view("uint16")
    return t.numpy()
