"""Device sampling (wgb_sample_rows) against the reference's host sampler.

The reference draws with an unseeded mt19937 (src/models/qwen2/model.cpp:
60-137), so a token is only comparable in distribution: the device's draws
must all lie in the kept set the oracle computes with the reference's rules
(oracle.sample_kept) and their frequencies must match the kept weights.
The CPU tests pin the oracle's kept set on hand-computed cases."""
import math

import numpy as np
import pytest
import torch

from oracle.oracle import sample_kept


def test_oracle_kept_set_by_hand():
    lg = np.log(np.array([1.0, 2.0, 4.0, 0.5], dtype=np.float64)).astype(np.float32)
    idx, w = sample_kept(lg, top_k=0, top_p=0.5, temperature=1.0)   # 4/7.5 >= 0.5
    assert idx.tolist() == [2]
    idx, w = sample_kept(lg, top_k=0, top_p=0.6, temperature=1.0)   # 4/7.5 < 0.6 <= 6/7.5
    assert idx.tolist() == [2, 1]
    idx, w = sample_kept(lg, top_k=3, top_p=1.0, temperature=1.0)
    assert idx.tolist() == [2, 1, 0]
    assert np.allclose(w / w.sum(), np.array([4, 2, 1]) / 7.0)
    idx, _ = sample_kept(lg, top_k=1, top_p=1.0, temperature=0.7)   # greedy
    assert idx.tolist() == [2]
    idx, _ = sample_kept(lg, top_k=5, top_p=2.0, temperature=-1.0)  # temperature <= 0: greedy
    assert idx.tolist() == [2]
    idx, _ = sample_kept(lg, top_k=-3, top_p=0.0, temperature=1.0)  # out-of-range k, p: all
    assert sorted(idx.tolist()) == [0, 1, 2, 3]


def test_oracle_ties_in_index_order():
    lg = np.array([1.0, 3.0, 3.0, 2.0, 3.0], dtype=np.float32)
    idx, _ = sample_kept(lg, top_k=2, top_p=1.0, temperature=1.0)
    assert idx.tolist() == [1, 2]


def test_oracle_temperature_sharpens():
    lg = np.array([0.0, 1.0], dtype=np.float32)
    _, w1 = sample_kept(lg, 0, 1.0, 1.0)
    _, w2 = sample_kept(lg, 0, 1.0, 0.25)
    assert w2[0] / w2.sum() > w1[0] / w1.sum()
    assert math.isclose(w2[1] / w2[0], math.exp(-4.0), rel_tol=1e-6)


# ---- device ------------------------------------------------------------------

CASES = [  # (top_k, top_p, temperature)
    (50, 1.0, 0.7), (0, 0.9, 1.0), (40, 0.8, 1.3), (5, 1.0, 1.0), (151936 * 2, 0.5, 0.8), (3, 0.3, 1.0),
]


def _draws(ops, logits_row, reps, k, p, t, seed):
    """reps draws of one logits row (one row per draw, one call)."""
    lg = logits_row.unsqueeze(0).repeat(reps, 1).contiguous()
    out = torch.empty(reps, dtype=torch.int64, device="cuda")
    ops.sample_rows(out, lg, k, p, t, seed=seed, offset=0)
    return out.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("k,p,t", CASES)
def test_sample_kept_set_and_frequencies(cuda, k, p, t):
    from wginfer_b200 import ops
    V = 151936
    g = torch.Generator().manual_seed(11)
    row = (torch.randn(V, generator=g) * 3.0).float()
    row[:8] += 12.0  # a few dominant tokens so that the kept sets are small and frequencies testable
    idx, w = sample_kept(row.numpy(), k, p, t)
    prob = dict(zip(idx.tolist(), (w / w.sum()).tolist()))
    n = 4096
    got = np.concatenate([_draws(ops, row.cuda(), 1024, k, p, t, seed=s) for s in range(4)])
    assert set(got.tolist()) <= set(prob), sorted(set(got.tolist()) - set(prob))[:5]
    vals, cnt = np.unique(got, return_counts=True)
    for tok, c in zip(vals.tolist(), cnt.tolist()):
        e = n * prob[tok]
        assert abs(c - e) <= 5 * math.sqrt(e * (1 - prob[tok])) + 3, (tok, c, e)
    # tokens the oracle gives at least 5% must appear
    for tok, q in prob.items():
        if q >= 0.05:
            assert tok in vals


@pytest.mark.gpu
def test_sample_greedy_cases_are_argmax(cuda):
    from wginfer_b200 import ops
    g = torch.Generator().manual_seed(3)
    lg = torch.randn(6, 1000, generator=g).cuda()
    want = lg.argmax(dim=1)
    out = torch.empty(6, dtype=torch.int64, device="cuda")
    for k, p, t in ((50, 0.9, 0.0), (1, 1.0, 0.8), (7, 0.5, -2.0)):
        ops.sample_rows(out, lg, k, p, t, seed=9)
        assert torch.equal(out, want)


@pytest.mark.gpu
def test_sample_reproducible_and_rows_differ(cuda):
    from wginfer_b200 import ops
    lg = torch.zeros(512, 300, device="cuda")  # uniform: every row a fresh draw
    a = torch.empty(512, dtype=torch.int64, device="cuda")
    b = torch.empty_like(a)
    ops.sample_rows(a, lg, 0, 1.0, 1.0, seed=5, offset=2)
    ops.sample_rows(b, lg, 0, 1.0, 1.0, seed=5, offset=2)
    assert torch.equal(a, b)
    ops.sample_rows(b, lg, 0, 1.0, 1.0, seed=5, offset=3)
    assert not torch.equal(a, b)
    assert len(set(a.tolist())) > 200
    assert int(a.min()) >= 0 and int(a.max()) < 300


@pytest.mark.gpu
def test_sample_bf16_ties_and_nan(cuda):
    """bf16 logits tie often: the k kept are the largest, ties by index."""
    from wginfer_b200 import ops
    row = torch.tensor([1.0, 5.0, 5.0, 2.0, 5.0, float("nan"), 4.0], dtype=torch.bfloat16)
    idx, _ = sample_kept(row.float().numpy(), 2, 1.0, 1.0)
    assert idx.tolist() == [1, 2]
    got = _draws(ops, row.cuda(), 2048, 2, 1.0, 1.0, seed=1)
    assert set(got.tolist()) == {1, 2}
    got = _draws(ops, row.cuda(), 2048, 0, 1.0, 1.0, seed=2)
    assert 5 not in set(got.tolist())  # NaN is never drawn
