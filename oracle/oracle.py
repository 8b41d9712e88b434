"""ctypes bindings for the two CPU checkers. TEST INFRASTRUCTURE ONLY.

* ``Oracle`` loads ``oracle/liboracle.so`` (our C restatement of the reference
  CPU path, oracle/wgo.c).
* ``Reference`` loads ``oracle/_ref/libwginfer_ref.so`` (the reference's own
  CPU sources compiled by oracle/Makefile), when it has been built.

Both expose the same numpy-level interface, so a test can run an input through
either and compare bits. Only tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU-baseline leg import this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libwginfer_ref.so")

DT_F16, DT_F32, DT_BF16, DT_I64 = 12, 13, 15, 6
_NP = {DT_F32: np.float32, DT_BF16: np.uint16, DT_F16: np.uint16}


def build(reference_root: str | None = None, quiet: bool = True) -> None:
    """Build liboracle.so, and the reference library when its source tree is
    given (the argument, else the WGINFER_REF_ROOT environment variable) and
    exists."""
    out = subprocess.DEVNULL if quiet else None
    subprocess.check_call(["make", "-C", HERE, "oracle"], stdout=out)
    ref = reference_root or os.environ.get("WGINFER_REF_ROOT")
    if ref and os.path.isdir(os.path.join(ref, "src")):
        subprocess.check_call(["make", "-C", HERE, "ref", f"REF={ref}"], stdout=out)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bits, as the reference's types.cpp:74-83."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class _Meta(C.Structure):
    _fields_ = [("dtype", C.c_int)] + [(n, C.c_size_t) for n in
                ("nlayer", "hs", "nh", "nkvh", "dh", "di", "maxseq", "voc")] + [
                ("epsilon", C.c_float), ("theta", C.c_float), ("end_token", C.c_int64)]


class _OpsBase:
    prefix = ""

    def __init__(self, path: str):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = C.CDLL(path)
        self.path = path
        for name in ("add", "argmax", "embedding", "linear", "rms_norm", "rope",
                     "self_attention", "swiglu"):
            fn = getattr(self.lib, self.prefix + name)
            fn.restype = C.c_int

    def _chk(self, rc, what):
        if rc != 0:
            raise RuntimeError(f"{self.prefix}{what} failed with status {rc}")

    # every op takes/returns numpy arrays; the caller allocates outputs
    def add(self, c, a, b, dt):
        self._chk(getattr(self.lib, self.prefix + "add")(_p(c), _p(a), _p(b), dt, C.c_size_t(a.size)), "add")

    def argmax(self, vals, dt):
        idx = np.zeros(1, np.int64)
        val = np.zeros(1, _NP[dt])
        self._chk(getattr(self.lib, self.prefix + "argmax")(_p(idx), _p(val), _p(vals), dt,
                                                          C.c_size_t(vals.size)), "argmax")
        return int(idx[0]), val[0]

    def linear(self, out, x, w, b, dt):
        M, K = x.shape
        N = w.shape[0]
        self._chk(getattr(self.lib, self.prefix + "linear")(_p(out), _p(x), _p(w), _p(b), dt,
                                                          C.c_size_t(M), C.c_size_t(N), C.c_size_t(K)), "linear")

    def rms_norm(self, out, x, w, eps, dt):
        M, N = x.shape
        self._chk(getattr(self.lib, self.prefix + "rms_norm")(_p(out), _p(x), _p(w), dt, C.c_size_t(M),
                                                            C.c_size_t(N), C.c_float(eps)), "rms_norm")

    def rope(self, out, x, pos, theta, dt):
        S, H, D = x.shape
        self._chk(getattr(self.lib, self.prefix + "rope")(_p(out), _p(x), _p(pos), dt, C.c_size_t(S),
                                                        C.c_size_t(H), C.c_size_t(D), C.c_float(theta)), "rope")

    def self_attention(self, out, q, k, v, scale, dt):
        S, NH, D = q.shape
        L, NKV, DV = v.shape
        self._chk(getattr(self.lib, self.prefix + "self_attention")(
            _p(out), _p(q), _p(k), _p(v), dt, C.c_size_t(S), C.c_size_t(NH), C.c_size_t(NKV),
            C.c_size_t(D), C.c_size_t(DV), C.c_size_t(L), C.c_float(scale)), "self_attention")

    def swiglu(self, out, g, u, dt):
        self._chk(getattr(self.lib, self.prefix + "swiglu")(_p(out), _p(g), _p(u), dt,
                                                          C.c_size_t(g.size)), "swiglu")


class Oracle(_OpsBase):
    prefix = "wgo_"

    def __init__(self, path: str = ORACLE_SO):
        super().__init__(path)
        self.lib.wgo_qwen2_create.restype = C.c_void_p
        self.lib.wgo_qwen2_infer.restype = C.c_int

    def embedding(self, out, idx, w, dt):
        self._chk(self.lib.wgo_embedding(_p(out), _p(idx), _p(w), dt, C.c_size_t(idx.size),
                                         C.c_size_t(w.shape[1]), C.c_size_t(w.shape[0])), "embedding")


class Reference(_OpsBase):
    prefix = "ref_"

    def __init__(self, path: str = REF_SO):
        super().__init__(path)
        self.lib.ref_qwen2_create.restype = C.c_void_p
        self.lib.ref_last_error.restype = C.c_char_p

    def embedding(self, out, idx, w, dt):
        self._chk(self.lib.ref_embedding(_p(out), _p(idx), _p(w), dt, C.c_size_t(idx.size),
                                         C.c_size_t(w.shape[1])), "embedding")


LAYER_NAMES = ("attn_norm_w", "attn_q_w", "attn_q_b", "attn_k_w", "attn_k_b", "attn_v_w",
               "attn_v_b", "attn_o_w", "mlp_norm_w", "mlp_gate_w", "mlp_up_w", "mlp_down_w")


class OracleQwen2:
    """The oracle's Qwen2 decoder over host weight arrays (dict of numpy)."""

    def __init__(self, ora: Oracle, meta: dict, weights: dict):
        self.ora, self.meta, self.w = ora, meta, weights
        m = _Meta(meta["dtype"], *[meta[k] for k in ("nlayer", "hs", "nh", "nkvh", "dh", "di",
                                                       "maxseq", "voc")],
                  meta["epsilon"], meta["theta"], meta.get("end_token", -1))
        L = meta["nlayer"]
        self._tables = {}
        fields = []
        for n in LAYER_NAMES:
            arr = (C.c_void_p * L)(*[_p(weights[n][l]) if weights[n][l] is not None else None
                                     for l in range(L)])
            self._tables[n] = arr
        class _W(C.Structure):
            _fields_ = [(n, C.c_void_p) for n in ("in_embed", "out_embed", "out_norm_w")] + [
                (n, C.c_void_p) for n in LAYER_NAMES]
        wstruct = _W(_p(weights["in_embed"]), _p(weights["out_embed"]), _p(weights["out_norm_w"]),
                     *[C.cast(self._tables[n], C.c_void_p) for n in LAYER_NAMES])
        self._wstruct = wstruct
        self.h = ora.lib.wgo_qwen2_create(C.byref(m), C.byref(wstruct))
        if not self.h:
            raise RuntimeError("wgo_qwen2_create failed")

    def reset(self):
        self.ora.lib.wgo_qwen2_reset_cache(C.c_void_p(self.h))

    def infer(self, ids, want_logits=False):
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        nxt = np.zeros(1, np.int64)
        lg = np.zeros(self.meta["voc"], np.float32) if want_logits else None
        rc = self.ora.lib.wgo_qwen2_infer(C.c_void_p(self.h), _p(ids), C.c_size_t(ids.size),
                                          _p(lg), _p(nxt))
        if rc:
            raise RuntimeError(f"wgo_qwen2_infer failed ({rc})")
        return (int(nxt[0]), lg) if want_logits else int(nxt[0])

    def __del__(self):
        if getattr(self, "h", None):
            self.ora.lib.wgo_qwen2_destroy(C.c_void_p(self.h))
            self.h = None


class ReferenceQwen2:
    """The reference's own Model (CPU device) fed the same host weights."""

    def __init__(self, ref: Reference, meta: dict, weights: dict):
        self.ref = ref
        m = _Meta(meta["dtype"], *[meta[k] for k in ("nlayer", "hs", "nh", "nkvh", "dh", "di",
                                                       "maxseq", "voc")],
                  meta["epsilon"], meta["theta"], meta.get("end_token", -1))
        self.h = ref.lib.ref_qwen2_create(C.byref(m))
        if not self.h:
            raise RuntimeError(ref.lib.ref_last_error().decode())
        def put(name, layer, arr):
            shape = (C.c_size_t * arr.ndim)(*arr.shape)
            rc = ref.lib.ref_qwen2_set_weight(C.c_void_p(self.h), name.encode(), layer, _p(arr),
                                              shape, arr.ndim)
            if rc:
                raise RuntimeError(ref.lib.ref_last_error().decode())
        for n in ("in_embed", "out_embed", "out_norm_w"):
            put(n, -1, weights[n])
        for n in LAYER_NAMES:
            for l in range(meta["nlayer"]):
                if weights[n][l] is not None:
                    put(n, l, weights[n][l])

    def reset(self):
        self.ref.lib.ref_qwen2_reset_cache(C.c_void_p(self.h))

    def infer(self, ids):
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        nxt = np.zeros(1, np.int64)
        rc = self.ref.lib.ref_qwen2_infer(C.c_void_p(self.h), _p(ids), C.c_size_t(ids.size), _p(nxt))
        if rc:
            raise RuntimeError(self.ref.lib.ref_last_error().decode())
        return int(nxt[0])

    def __del__(self):
        if getattr(self, "h", None):
            self.ref.lib.ref_qwen2_destroy(C.c_void_p(self.h))
            self.h = None


def sample_kept(logits: np.ndarray, top_k: int, top_p: float, temperature: float):
    """The kept set of the reference's host sampler, sample_from_logits
    (src/models/qwen2/model.cpp:60-137), for f32 logits: (indices in
    decreasing logit order, their weights). Logits that compare equal are
    taken in index order (the reference's partial_sort leaves them in an
    unspecified order). temperature <= 0 or top_k == 1 with top_p >= 1 give
    the argmax alone (weight 1)."""
    lg = np.asarray(logits, dtype=np.float32).reshape(-1)
    vocab = lg.size
    if not temperature > 0.0:
        return np.array([int(np.argmax(lg))]), np.array([1.0])
    if top_k <= 0 or top_k > vocab:
        top_k = vocab
    if not top_p > 0.0 or top_p > 1.0:
        top_p = 1.0
    if top_k == 1 and top_p >= 1.0:
        return np.array([int(np.argmax(lg))]), np.array([1.0])
    order = np.argsort(-lg, kind="stable")[:top_k]          # model.cpp:84-93
    inv_temp = np.float32(1.0) / np.float32(temperature)    # :96
    scaled = (lg[order] * inv_temp).astype(np.float32)
    max_scaled = scaled.max()                               # :97-100
    probs = np.exp((scaled - max_scaled).astype(np.float32).astype(np.float64))  # :103-111
    probs[~np.isfinite(probs) | (probs < 0)] = 0.0
    total = 0.0
    for p in probs:
        total += p
    if top_p < 1.0:                                         # :117-130
        cum, keep = 0.0, 0
        tp = float(np.float32(top_p))
        for i, p in enumerate(probs):
            cum += p / total
            keep = i + 1
            if cum >= tp:
                break
        keep = max(keep, 1)
        order, probs = order[:keep], probs[:keep]
    return order, probs

