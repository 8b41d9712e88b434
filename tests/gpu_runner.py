"""Runs the parity cases through the B200 backend's C-ABI (wginfer_b200.ops)
with the oracle's numpy interface, so a test can diff the two."""
import numpy as np
import torch

from wginfer_b200 import ops

_TD = {13: torch.float32, 15: torch.bfloat16, 12: torch.float16}


def to_dev(a, dt=None):
    if a is None:
        return None
    if a.dtype == np.int64:
        return torch.from_numpy(a).cuda()
    if a.dtype == np.float32:
        return torch.from_numpy(a).cuda()
    t = torch.from_numpy(a.view(np.int16)).cuda()
    return t.view(_TD[dt])


def to_host(t, like):
    t = t.detach().cpu()
    if like.dtype == np.float32:
        return t.numpy().astype(np.float32)
    if like.dtype == np.int64:
        return t.numpy().astype(np.int64)
    return t.view(torch.int16).numpy().view(np.uint16).reshape(like.shape)


class Gpu:
    """Same method signatures as oracle.Oracle; outputs are filled in place."""

    def add(self, c, a, b, dt):
        C = to_dev(c, dt)
        ops.add(C, to_dev(a, dt), to_dev(b, dt))
        c[...] = to_host(C, c)

    def swiglu(self, o, g, u, dt):
        O = to_dev(o, dt)
        ops.swiglu(O, to_dev(g, dt), to_dev(u, dt))
        o[...] = to_host(O, o)

    def rms_norm(self, o, x, w, eps, dt):
        O = to_dev(o, dt)
        ops.rms_norm(O, to_dev(x, dt), to_dev(w, dt), eps)
        o[...] = to_host(O, o)

    def rope(self, o, x, pos, theta, dt):
        O = to_dev(o, dt)
        ops.rope(O, to_dev(x, dt), to_dev(pos), theta)
        o[...] = to_host(O, o)

    def linear(self, o, x, w, b, dt):
        O = to_dev(o, dt)
        ops.linear(O, to_dev(x, dt), to_dev(w, dt), to_dev(b, dt))
        o[...] = to_host(O, o)

    def self_attention(self, o, q, k, v, scale, dt):
        O = to_dev(o, dt)
        ops.self_attention(O, to_dev(q, dt), to_dev(k, dt), to_dev(v, dt), scale)
        o[...] = to_host(O, o)

    def argmax(self, vals, dt):
        V = to_dev(vals, dt) if vals.size else torch.empty(0, dtype=_TD[dt], device="cuda")
        idx = torch.zeros(1, dtype=torch.int64, device="cuda")
        val = torch.zeros(1, dtype=_TD[dt], device="cuda")
        ops.argmax(idx, val, V)
        like = np.zeros(1, np.float32 if dt == 13 else np.uint16)
        return int(idx.item()), to_host(val, like)[0]

    def embedding(self, o, idx, w, dt):
        O = to_dev(o, dt)
        ops.embedding(O, to_dev(idx), to_dev(w, dt))
        o[...] = to_host(O, o)
