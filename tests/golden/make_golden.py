"""Generates the committed golden fixtures from the reference's own CPU code.

Run from the repo root, in a container where the reference tree exists
(oracle/_ref/libwginfer_ref.so is built from it by oracle/Makefile):

    python tests/golden/make_golden.py            # ops + small models
    python tests/golden/make_golden.py --full     # + 28-layer token streams
    python tests/golden/make_golden.py --skip-ops --only NAME ...   # selected streams

Inputs are regenerated from seeds by tests/golden/cases.py, so only outputs
are stored: bits for small outputs, SHA-256 of the bits for large ones.
Op outputs come from the reference build (oracle/_ref); the 28-layer Qwen2
streams come from the oracle restatement (the reference takes ~18 s per token
there) after its first tokens were checked against the reference itself. The
batched streams (64 sequences with 2048-token prompts on the one-layer model)
come from the oracle, decoding each checked sequence on its own (sequences in
a batch are independent); the reference would take about 15 minutes per
2048-token prefill because it forms logits for every prompt row.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from tests.golden import cases as CS  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
SMALL = 4096  # outputs up to this many bytes are stored in full


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def ops_golden(ref) -> None:
    index, blobs = [], {}
    for i, case in enumerate(CS.OP_CASES):
        outs = CS.run_case(ref, case)
        entry = {"id": i, **{k: v for k, v in case.items()}}
        entry["outputs"] = []
        for j, o in enumerate(outs):
            o = np.ascontiguousarray(o)
            e = {"sha256": digest(o), "dtype": str(o.dtype), "shape": list(o.shape)}
            if o.nbytes <= SMALL:
                blobs[f"c{i}_o{j}"] = o
                e["stored"] = f"c{i}_o{j}"
            entry["outputs"].append(e)
        index.append(entry)
    np.savez_compressed(os.path.join(HERE, "ops_golden.npz"), **blobs)
    with open(os.path.join(HERE, "ops_golden.json"), "w") as f:
        json.dump(index, f, indent=1)
    print(f"ops: {len(index)} cases")


def model_stream(model_cls, lib, cfg, prompt_len, steps, seed=0, logits=False):
    meta, w = CS.model_inputs(cfg, seed)
    m = model_cls(lib, meta, w)
    ids = CS.prompt(prompt_len, cfg.voc, seed)
    toks, margins = [], []
    if logits:
        t, lg = m.infer(ids, want_logits=True)
    else:
        t = m.infer(ids)
    toks.append(t)
    if logits:
        margins.append(CS.top2_margin(lg))
    for _ in range(steps - 1):
        if logits:
            t, lg = m.infer(np.array([t]), want_logits=True)
            margins.append(CS.top2_margin(lg))
        else:
            t = m.infer(np.array([t]))
        toks.append(t)
    return toks, margins


def batched_golden(ora, name, spec):
    meta, w = CS.model_inputs(spec["cfg"], 0)
    ids = CS.batched_prompts(spec)
    streams, margins = {}, {}
    for seq in spec["checked"]:
        m = O.OracleQwen2(ora, meta, w)
        t, lg = m.infer(ids[seq], want_logits=True)
        toks, mg = [t], [CS.top2_margin(lg)]
        for _ in range(spec["steps"] - 1):
            t, lg = m.infer(np.array([t]), want_logits=True)
            toks.append(t)
            mg.append(CS.top2_margin(lg))
        streams[str(seq)], margins[str(seq)] = toks, mg
        del m
    return {"streams": streams, "margins": margins,
            "source": "oracle, each checked sequence decoded on its own"}


def models_golden(ref, ora, full: bool, only=None) -> None:
    path = os.path.join(HERE, "qwen2_streams.json")
    out = json.load(open(path)) if os.path.exists(path) else {}
    for name, spec in CS.BATCHED.items():
        if only is not None and name not in only:
            continue
        t0 = time.time()
        out[name] = batched_golden(ora, name, spec)
        print(f"{name}: {len(spec['checked'])} streams in {time.time() - t0:.1f}s", flush=True)
        with open(path, "w") as f:
            json.dump(out, f, indent=1)
    for name, (cfg, plen, steps) in CS.SMALL_MODELS.items():
        if only is not None and name not in only:
            continue
        t0 = time.time()
        rt, _ = model_stream(O.ReferenceQwen2, ref, cfg, plen, steps)
        ot, om = model_stream(O.OracleQwen2, ora, cfg, plen, steps, logits=True)
        assert rt == ot, f"oracle and reference disagree on {name}: {rt} vs {ot}"
        out[name] = {"tokens": rt, "margins": om, "source": "reference (oracle agrees)"}
        print(f"{name}: {len(rt)} tokens in {time.time() - t0:.1f}s", flush=True)
    if full:
        for name, (cfg, plen, steps, ref_prefix) in CS.FULL_MODELS.items():
            if only is not None and name not in only:
                continue
            t0 = time.time()
            ot, om = model_stream(O.OracleQwen2, ora, cfg, plen, steps, logits=True)
            rt, _ = model_stream(O.ReferenceQwen2, ref, cfg, plen, ref_prefix) if ref_prefix else ([], [])
            assert ot[:len(rt)] == rt, f"oracle and reference disagree on {name} prefix: {ot[:len(rt)]} vs {rt}"
            out[name] = {"tokens": ot, "margins": om,
                         "source": f"oracle; first {len(rt)} tokens checked against the reference"}
            print(f"{name}: {len(ot)} tokens in {time.time() - t0:.1f}s", flush=True)
            with open(path, "w") as f:
                json.dump(out, f, indent=1)
    with open(path, "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--full", action="store_true")
    ap.add_argument("--skip-ops", action="store_true")
    ap.add_argument("--only", nargs="*", default=None, help="stream names to (re)generate")
    ap.add_argument("--reference-root", default=None, help="reference source tree (for oracle/_ref)")
    a = ap.parse_args()
    O.build(a.reference_root)
    ref, ora = O.Reference(), O.Oracle()
    if not a.skip_ops:
        ops_golden(ref)
    models_golden(ref, ora, a.full or bool(a.only), a.only)
