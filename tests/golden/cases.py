"""Seeded parity cases shared by the golden generator and the tests.

Inputs are drawn from torch's CPU generator (bit-reproducible for a given
torch build) and rounded to the case dtype, then handed to a runner as
numpy arrays of raw bits (f32 as float32, bf16/f16 as uint16). Shapes follow
the reference's own op tests (test/ops/*.py) and the decode-path shapes of
Qwen2-1.5B (hidden 1536, 12/2 heads of 128, MLP 8960, vocab 151936),
including ragged sizes, single rows/keys, empty inputs and fully masked
attention rows.
"""
from __future__ import annotations

import numpy as np
import torch

from wginfer_b200.synthetic import Qwen2Config, qwen2_weights, to_numpy_bits

DT = {"f32": 13, "bf16": 15, "f16": 12}
TORCH_DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def draw(shape, dtype: str, seed: int, std=1.0, mean=0.0):
    g = torch.Generator("cpu").manual_seed(seed)
    t = torch.randn(tuple(shape), generator=g, dtype=torch.float32) * std + mean
    return to_numpy_bits(t.to(TORCH_DT[dtype]))


def out_like(shape, dtype: str):
    return np.zeros(tuple(shape), np.float32 if dtype == "f32" else np.uint16)


OP_CASES = [
    # the config-1 op chain (f32, T = 16, hidden 1536)
    dict(op="rms_norm", dtype="f32", M=16, N=1536, eps=1e-6, seed=11),
    dict(op="rope", dtype="f32", S=16, H=12, D=128, p0=0, theta=1e4, seed=12),
    dict(op="rope", dtype="f32", S=16, H=2, D=128, p0=0, theta=1e4, seed=13),
    dict(op="swiglu", dtype="f32", shape=[16, 8960], seed=14),
    dict(op="add", dtype="f32", shape=[16, 1536], seed=15),
    dict(op="linear", dtype="f32", M=16, N=1536, K=1536, bias=True, seed=16),
    dict(op="argmax", dtype="f32", n=151936, seed=17),
    # reference test shapes and edges
    dict(op="add", dtype="f32", shape=[2, 3], seed=20),
    dict(op="add", dtype="bf16", shape=[2, 3], seed=21),
    dict(op="add", dtype="bf16", shape=[1001], seed=22),
    dict(op="add", dtype="f16", shape=[4099], seed=23),
    dict(op="swiglu", dtype="bf16", shape=[3, 8960], seed=24),
    dict(op="swiglu", dtype="bf16", shape=[1, 7], seed=25),
    dict(op="rms_norm", dtype="f32", M=1, N=4, eps=1e-5, seed=26),
    dict(op="rms_norm", dtype="bf16", M=1, N=1536, eps=1e-6, seed=27),
    dict(op="rms_norm", dtype="bf16", M=5, N=4096, eps=1e-6, seed=28),
    dict(op="rms_norm", dtype="bf16", M=3, N=100, eps=1e-6, seed=29),
    dict(op="rope", dtype="f32", S=2, H=1, D=4, p0=0, theta=1e4, seed=30),
    dict(op="rope", dtype="bf16", S=1, H=12, D=128, p0=700, theta=1e4, seed=31),
    dict(op="rope", dtype="bf16", S=3, H=2, D=128, p0=2300, theta=1e6, seed=32),
    dict(op="linear", dtype="f32", M=2, N=3, K=4, bias=True, seed=33),
    dict(op="linear", dtype="f32", M=2, N=3, K=4, bias=False, seed=34),
    dict(op="linear", dtype="bf16", M=1, N=2048, K=1536, bias=True, seed=35),
    dict(op="linear", dtype="bf16", M=1, N=1536, K=8960, bias=False, seed=36),
    dict(op="linear", dtype="bf16", M=4, N=300, K=1536, bias=True, seed=37),
    dict(op="linear", dtype="bf16", M=3, N=37, K=100, bias=True, seed=38),
    dict(op="linear", dtype="bf16", M=20, N=256, K=1536, bias=True, seed=39),
    dict(op="self_attention", dtype="f32", S=2, L=2, nh=1, nkvh=1, d=4, seed=40),
    dict(op="self_attention", dtype="f32", S=5, L=11, nh=4, nkvh=2, d=8, seed=41),
    dict(op="self_attention", dtype="bf16", S=1, L=37, nh=12, nkvh=2, d=128, seed=42),
    dict(op="self_attention", dtype="bf16", S=1, L=640, nh=12, nkvh=2, d=128, seed=43),
    dict(op="self_attention", dtype="bf16", S=16, L=16, nh=12, nkvh=2, d=128, seed=44),
    dict(op="self_attention", dtype="bf16", S=7, L=3, nh=4, nkvh=2, d=8, seed=45),
    dict(op="self_attention", dtype="bf16", S=1, L=1, nh=12, nkvh=2, d=128, seed=46),
    dict(op="argmax", dtype="bf16", n=151936, seed=47),
    dict(op="argmax", dtype="bf16", n=4, seed=48),
    dict(op="argmax", dtype="f16", n=4096, seed=49),
    dict(op="argmax", dtype="bf16", n=1000, seed=50, ties=True),
    dict(op="argmax", dtype="f32", n=0, seed=51),
    dict(op="embedding", dtype="bf16", T=50, V=512, D=64, seed=52),
    dict(op="embedding", dtype="f32", T=1, V=2, D=3, seed=53),
    dict(op="embedding", dtype="bf16", T=4, V=151936, D=1536, seed=54),
]


def inputs(case):
    """Input arrays of a case, in the runner's argument order."""
    op, dt, s = case["op"], case["dtype"], case["seed"]
    if op in ("add", "swiglu"):
        return [draw(case["shape"], dt, s), draw(case["shape"], dt, s + 1000)]
    if op == "rms_norm":
        return [draw([case["M"], case["N"]], dt, s), draw([case["N"]], dt, s + 1000, std=0.1, mean=1.0)]
    if op == "rope":
        pos = np.arange(case["p0"], case["p0"] + case["S"], dtype=np.int64)
        return [draw([case["S"], case["H"], case["D"]], dt, s), pos]
    if op == "linear":
        x = draw([case["M"], case["K"]], dt, s)
        w = draw([case["N"], case["K"]], dt, s + 1000, std=0.02)
        b = draw([case["N"]], dt, s + 2000, std=0.02) if case["bias"] else None
        return [x, w, b]
    if op == "self_attention":
        q = draw([case["S"], case["nh"], case["d"]], dt, s)
        k = draw([case["L"], case["nkvh"], case["d"]], dt, s + 1000)
        v = draw([case["L"], case["nkvh"], case["d"]], dt, s + 2000)
        return [q, k, v]
    if op == "argmax":
        v = draw([case["n"]], dt, s)
        if case.get("ties") and case["n"] > 10:
            # equal maxima at 3, 500, 999 (and wherever the maximum was): the first must win
            mx = int(np.argmax(_as_f32(v, dt)))
            v[[3, 500, 999]] = v[mx]
        return [v]
    if op == "embedding":
        w = draw([case["V"], case["D"]], dt, s)
        g = torch.Generator("cpu").manual_seed(s + 1000)
        idx = torch.randint(0, case["V"], (case["T"],), generator=g, dtype=torch.int64).numpy()
        return [idx, w]
    raise ValueError(op)


def _as_f32(a, dt):
    if dt == "f32":
        return a.astype(np.float32)
    if dt == "bf16":
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.view(np.float16).astype(np.float32)


def run_case(lib, case, ins=None):
    """Runs a case on an ops object with the oracle.Oracle/Reference interface."""
    op, dt = case["op"], case["dtype"]
    d = DT[dt]
    ins = inputs(case) if ins is None else ins
    if op == "add":
        out = out_like(case["shape"], dt)
        lib.add(out, ins[0], ins[1], d)
        return [out]
    if op == "swiglu":
        out = out_like(case["shape"], dt)
        lib.swiglu(out, ins[0], ins[1], d)
        return [out]
    if op == "rms_norm":
        out = out_like([case["M"], case["N"]], dt)
        lib.rms_norm(out, ins[0], ins[1], case["eps"], d)
        return [out]
    if op == "rope":
        out = out_like([case["S"], case["H"], case["D"]], dt)
        lib.rope(out, ins[0], ins[1], case["theta"], d)
        return [out]
    if op == "linear":
        out = out_like([case["M"], case["N"]], dt)
        lib.linear(out, ins[0], ins[1], ins[2], d)
        return [out]
    if op == "self_attention":
        out = out_like([case["S"], case["nh"], case["d"]], dt)
        lib.self_attention(out, ins[0], ins[1], ins[2], 1.0 / float(np.sqrt(case["d"])), d)
        return [out]
    if op == "argmax":
        idx, val = lib.argmax(ins[0], d)
        return [np.array([idx], np.int64), np.array([val], np.float32 if dt == "f32" else np.uint16)]
    if op == "embedding":
        out = out_like([case["T"], case["D"]], dt)
        lib.embedding(out, ins[0], ins[1], d)
        return [out]
    raise ValueError(op)


# ---- Qwen2 token streams -------------------------------------------------
TINY = Qwen2Config(nlayer=2, hs=256, nh=4, nkvh=2, dh=64, di=512, voc=1000, maxseq=256)
ONE_LAYER = Qwen2Config(nlayer=1, maxseq=640)          # the config-2 layer with embeddings and lm_head
ONE_LAYER_2K = Qwen2Config(nlayer=1, maxseq=2048 + 256)  # the same model with room for 2048-token prompts
FULL = Qwen2Config(nlayer=28, maxseq=640)              # Qwen2-1.5B architecture

# name -> (config, prompt length, generated tokens)
SMALL_MODELS = {
    "tiny_p16_g64": (TINY, 16, 64),
    "tiny_p100_g32": (TINY, 100, 32),
    "one_layer_p16_g12": (ONE_LAYER, 16, 12),
    # one decoder layer, 512-token prefill, 128 decode steps
    "one_layer_p512_g128": (ONE_LAYER, 512, 128),
}

# Batched decode: 64 sequences with uniform random 2048-token prompts (ids
# from prompt_ids(2048, voc, seed=prompt_seed, batch=64)) decoded together on
# the one-layer model; the streams of the `checked` sequences are stored.
BATCHED = {
    "one_layer_bs64_p2048": dict(cfg=ONE_LAYER_2K, prompt=2048, sequences=64, prompt_seed=1000,
                                 checked=[0, 21, 42, 63], steps=16),
}


def batched_prompts(spec) -> np.ndarray:
    from wginfer_b200.synthetic import prompt_ids
    return prompt_ids(spec["prompt"], spec["cfg"].voc, seed=spec["prompt_seed"], batch=spec["sequences"]).numpy()
# name -> (config, prompt length, generated tokens, tokens checked against the reference itself)
FULL_MODELS = {
    "qwen2_1p5b_p16_g128": (FULL, 16, 128, 3),
    "qwen2_1p5b_p128_g128": (FULL, 128, 128, 0),
    "qwen2_1p5b_p512_g128": (FULL, 512, 128, 0),
}


def model_inputs(cfg: Qwen2Config, seed: int = 0):
    w = qwen2_weights(cfg, seed=seed)
    wn = {k: ([to_numpy_bits(x) if x is not None else None for x in v] if isinstance(v, list) else to_numpy_bits(v))
          for k, v in w.items()}
    meta = dict(dtype=15, nlayer=cfg.nlayer, hs=cfg.hs, nh=cfg.nh, nkvh=cfg.nkvh, dh=cfg.dh, di=cfg.di,
                maxseq=cfg.maxseq, voc=cfg.voc, epsilon=cfg.epsilon, theta=cfg.theta)
    return meta, wn


def prompt(n: int, voc: int, seed: int = 0) -> np.ndarray:
    from wginfer_b200.synthetic import prompt_ids
    return prompt_ids(n, voc, seed).numpy()


def top2_margin(logits: np.ndarray) -> float:
    top = np.partition(logits, -2)[-2:]
    return float(abs(top[1] - top[0]))
