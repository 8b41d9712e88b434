"""Qwen2 decoder on the B200 backend (wraps wgb_qwen2_* of the C-ABI).

Mirrors the reference's ``wginfer.models.Qwen2`` driver
(python/wginfer/models/qwen2.py:15-235): ``infer`` is ``Model::infer``,
``generate`` is the greedy loop with EOS stop. Weights come from a dict of
tensors with the reference's ModelWeights names (``synthetic.qwen2_weights``
produces one). ``prefill``/``decode_step`` expose the device-resident batched
path: one CUDA-graph launch per step, tokens stay on the device.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from .synthetic import LAYER_NAMES, Qwen2Config


class _Meta(C.Structure):
    _fields_ = [("dtype", C.c_int)] + [(n, C.c_size_t) for n in
                ("nlayer", "hs", "nh", "nkvh", "dh", "di", "maxseq", "voc")] + [
                ("epsilon", C.c_float), ("theta", C.c_float), ("end_token", C.c_int64)]


_DT = {torch.bfloat16: _lib.DT_BF16, torch.float32: _lib.DT_F32, torch.float16: _lib.DT_F16}


class Qwen2:
    def __init__(self, cfg: Qwen2Config, weights: dict | None = None, device: int = 0, max_batch: int = 1):
        self.cfg = cfg
        self.device = device
        self.max_batch = max_batch
        self._l = _lib.lib()
        meta = _Meta(_DT[cfg.dtype], cfg.nlayer, cfg.hs, cfg.nh, cfg.nkvh, cfg.dh, cfg.di, cfg.maxseq, cfg.voc,
                     cfg.epsilon, cfg.theta, cfg.end_token)
        h = C.c_void_p()
        _lib.check(self._l.wgb_qwen2_create(C.byref(meta), device, max_batch, C.byref(h)), "wgb_qwen2_create")
        self.h = h
        self._pinned = torch.empty(max(1, max_batch), dtype=torch.int64).pin_memory()
        self._init_call_buffers()
        if weights is not None:
            self.load_weights(weights)

    def _init_call_buffers(self) -> None:
        # one-token infer calls (every decode step) reuse these instead of
        # building a numpy array per call (about 3.5 us of host time each)
        self._tok = (C.c_int64 * 1)()
        self._next = C.c_int64(0)
        self._next_ref = C.byref(self._next)

    def set_weight(self, name: str, t: torch.Tensor, layer: int = -1) -> None:
        t = t.contiguous()
        on_host = t.device.type == "cpu"
        _lib.check(self._l.wgb_qwen2_set_weight(self.h, name.encode(), layer, C.c_void_p(t.data_ptr()),
                                                t.numel() * t.element_size(), int(on_host)), f"set_weight({name})")

    def load_weights(self, w: dict) -> None:
        for n in ("in_embed", "out_embed", "out_norm_w"):
            self.set_weight(n, w[n])
        for n in LAYER_NAMES:
            for l, t in enumerate(w[n]):
                if t is not None:
                    self.set_weight(n, t, l)

    def reset_cache(self) -> None:
        _lib.check(self._l.wgb_qwen2_reset_cache(self.h), "reset_cache")

    def infer(self, token_ids, top_k=1, top_p=1.0, temperature=1.0) -> int:
        """Model::infer for sequence 0: returns the next token (host int)."""
        if (type(token_ids) in (list, tuple) and len(token_ids) == 1 and type(token_ids[0]) is int
                and -(1 << 63) <= token_ids[0] < (1 << 63)):
            self._tok[0] = token_ids[0]
            _lib.check(self._l.wgb_qwen2_infer(self.h, self._tok, 1, top_k, top_p, temperature, self._next_ref),
                       "infer")
            return self._next.value
        ids = np.ascontiguousarray(np.asarray(token_ids, dtype=np.int64).reshape(-1))
        nxt = C.c_int64(0)
        _lib.check(self._l.wgb_qwen2_infer(self.h, ids.ctypes.data_as(C.c_void_p), ids.size, top_k, top_p,
                                           temperature, C.byref(nxt)), "infer")
        return int(nxt.value)

    def generate(self, prompt_ids, max_new_tokens=128, stop_at_eos=True) -> list[int]:
        """Greedy generation (python/wginfer/models/qwen2.py:168-195)."""
        self.reset_cache()
        out = []
        nxt = self.infer(prompt_ids)
        for _ in range(max_new_tokens):
            out.append(nxt)
            if stop_at_eos and self.cfg.end_token >= 0 and nxt == self.cfg.end_token:
                break
            if len(out) == max_new_tokens:
                break
            nxt = self.infer([nxt])
        return out

    # ---- device-resident batched path ----
    def prefill(self, seq: int, token_ids) -> None:
        ids = np.ascontiguousarray(np.asarray(token_ids, dtype=np.int64).reshape(-1))
        _lib.check(self._l.wgb_qwen2_prefill(self.h, seq, ids.ctypes.data_as(C.c_void_p), ids.size), "prefill")

    def decode_step(self, batch: int) -> None:
        _lib.check(self._l.wgb_qwen2_decode_step(self.h, batch), "decode_step")

    @property
    def stream_handle(self) -> int:
        return self._l.wgb_qwen2_stream(self.h) or 0

    def torch_stream(self) -> torch.cuda.ExternalStream:
        return torch.cuda.ExternalStream(self.stream_handle, device=torch.device("cuda", self.device))

    def tokens(self, batch: int) -> list[int]:
        """Current device tokens of sequences [0, batch) (synchronises)."""
        buf = np.zeros(batch, np.int64)
        _lib.check(self._l.wgb_qwen2_read_tokens(self.h, buf.ctypes.data_as(C.c_void_p), batch), "read_tokens")
        return buf.tolist()

    def trace_step(self, batch: int = 1):
        """Per-launch device times (us) of one eagerly launched decode step."""
        us = np.zeros(1024, np.float32)
        names = C.create_string_buffer(1 << 16)
        n = C.c_int(0)
        _lib.check(self._l.wgb_qwen2_trace_step(self.h, batch, 1024, us.ctypes.data_as(C.c_void_p), names,
                                                1 << 16, C.byref(n)), "trace_step")
        return list(zip(names.value.decode().split("\n")[:n.value], us[:n.value].tolist()))

    def cache_len(self, seq: int = 0) -> int:
        return int(self._l.wgb_qwen2_cache_len(self.h, seq))

    def logits(self, seq: int = 0) -> np.ndarray:
        """The last logits row of `seq`, widened to f32 on the host."""
        buf = np.zeros(self.cfg.voc, np.float32)
        _lib.check(self._l.wgb_qwen2_read_logits(self.h, seq, buf.ctypes.data_as(C.c_void_p)), "read_logits")
        return buf

    def close(self) -> None:
        if getattr(self, "h", None):
            self._l.wgb_qwen2_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
