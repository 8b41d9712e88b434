"""The CPU oracle pinned against the reference: committed golden fixtures
(made from the reference's own CPU build) and, where that build exists, the
reference live."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from tests.golden import cases as CS

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
GOLD = json.load(open(os.path.join(HERE, "ops_golden.json")))
BLOBS = np.load(os.path.join(HERE, "ops_golden.npz"))
STREAMS = json.load(open(os.path.join(HERE, "qwen2_streams.json")))


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("cid", range(len(CS.OP_CASES)))
def test_oracle_matches_golden(oracle, cid):
    case = CS.OP_CASES[cid]
    g = GOLD[cid]
    assert g["op"] == case["op"] and g["seed"] == case["seed"]
    outs = CS.run_case(oracle, case)
    for o, e in zip(outs, g["outputs"]):
        if "stored" in e:
            assert np.array_equal(o, BLOBS[e["stored"]])
        assert _sha(o) == e["sha256"], f"case {cid} {case}"


@pytest.mark.parametrize("cid", range(len(CS.OP_CASES)))
def test_oracle_matches_reference_live(oracle, reference, cid):
    case = CS.OP_CASES[cid]
    ins = CS.inputs(case)
    a = CS.run_case(oracle, case, ins)
    b = CS.run_case(reference, case, ins)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


@pytest.mark.parametrize("name", ["tiny_p16_g64", "tiny_p100_g32"])
def test_oracle_qwen2_stream(oracle, name):
    from oracle.oracle import OracleQwen2
    cfg, plen, steps = CS.SMALL_MODELS[name]
    meta, w = CS.model_inputs(cfg)
    m = OracleQwen2(oracle, meta, w)
    ids = CS.prompt(plen, cfg.voc)
    toks = [m.infer(ids)]
    for _ in range(steps - 1):
        toks.append(m.infer(np.array([toks[-1]])))
    assert toks == STREAMS[name]["tokens"]


def test_oracle_qwen2_matches_reference_live(oracle, reference):
    from oracle.oracle import OracleQwen2, ReferenceQwen2
    cfg = CS.TINY
    meta, w = CS.model_inputs(cfg, seed=3)
    a, b = OracleQwen2(oracle, meta, w), ReferenceQwen2(reference, meta, w)
    ids = CS.prompt(9, cfg.voc, seed=3)
    ta, tb = [a.infer(ids)], [b.infer(ids)]
    for _ in range(20):
        ta.append(a.infer(np.array([ta[-1]])))
        tb.append(b.infer(np.array([tb[-1]])))
    assert ta == tb


def test_bf16_rounding_matches_torch():
    from oracle.oracle import f32_to_bf16
    x = torch.randn(100000, generator=torch.Generator().manual_seed(5)) * 7
    x[:4] = torch.tensor([0.0, -0.0, 1e-40, 3.0e38])
    mine = f32_to_bf16(x.numpy())
    theirs = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(mine, theirs)


def test_oracle_rejects_bad_embedding_index(oracle):
    w = np.zeros((4, 8), np.float32)
    out = np.zeros((1, 8), np.float32)
    with pytest.raises(RuntimeError):
        oracle.embedding(out, np.array([4], np.int64), w, 13)
