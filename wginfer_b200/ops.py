"""Op front for the B200 backend: the reference's ``Ops.<op>`` surface over
torch CUDA tensors.

Each function repeats the validation of the reference's op front
(``src/ops/<op>/op.cpp``) with the same argument order and meaning, then calls
the C-ABI (include/wginfer_b200.h) on the current torch stream. Validation
failures the reference reports as ``std::invalid_argument`` raise
``ValueError``; its ``ASSERT`` failures (contiguity) raise ``RuntimeError``.
There is no CPU path: tensors must live on a CUDA device.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib

_DT = {torch.float32: _lib.DT_F32, torch.bfloat16: _lib.DT_BF16, torch.float16: _lib.DT_F16}


def _dt(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise RuntimeError(f"Unsupported dtype {t.dtype}") from None


def _stream(t: torch.Tensor):
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _same_device(*ts):
    d = ts[0].device
    for t in ts:
        if t.device != d:
            raise RuntimeError("device mismatch")
    if d.type != "cuda":
        raise RuntimeError("Unsupported device: the B200 backend runs on CUDA tensors only")


def _contig(msg, *ts):
    if not all(t.is_contiguous() for t in ts):
        raise RuntimeError(msg)


def _arg(cond, msg):
    if not cond:
        raise ValueError(msg)


def add(c, a, b):
    """src/ops/add/op.cpp:16-44."""
    _same_device(c, a, b)
    if not (c.shape == a.shape == b.shape):
        raise ValueError("Shapes mismatch")
    if not (c.dtype == a.dtype == b.dtype):
        raise ValueError("Datatypes mismatch")
    _contig("Add: all tensors must be contiguous.", c, a, b)
    with torch.cuda.device(c.device):
        _lib.check(_lib.lib().wgb_add(_ptr(c), _ptr(a), _ptr(b), _dt(c), c.numel(), _stream(c)), "add")


def argmax(max_idx, max_val, vals):
    """src/ops/argmax/op.cpp:15-56."""
    _same_device(max_idx, max_val, vals)
    _arg(vals.dim() == 1, "vals only support 1D tensor for now")
    _arg(max_idx.dim() == 1 and max_idx.numel() == 1, "max_idx should be a single element")
    _arg(max_val.dim() == 1 and max_val.numel() == 1, "max_val should be a single element")
    if max_idx.dtype != torch.int64 or max_val.dtype != vals.dtype:
        raise ValueError("Datatypes mismatch")
    _contig("max_idx, max_val and vals must be contiguous", max_idx, max_val, vals)
    with torch.cuda.device(vals.device):
        _lib.check(_lib.lib().wgb_argmax(_ptr(max_idx), _ptr(max_val), _ptr(vals), _dt(vals), vals.numel(),
                                         _stream(vals)), "argmax")


def argmax_rows(max_idx, max_val, vals):
    """Batched argmax over vals[B, V] (new entry for batched decode)."""
    _same_device(max_idx, vals)
    _arg(vals.dim() == 2, "vals must be 2D [rows, n]")
    _arg(max_idx.numel() == vals.shape[0] and max_idx.dtype == torch.int64, "max_idx must be int64 [rows]")
    if max_val is not None:
        _arg(max_val.numel() == vals.shape[0] and max_val.dtype == vals.dtype, "max_val must be [rows] of vals' dtype")
    _contig("tensors must be contiguous", max_idx, vals)
    with torch.cuda.device(vals.device):
        _lib.check(_lib.lib().wgb_argmax_rows(_ptr(max_idx), _ptr(max_val), _ptr(vals), _dt(vals), vals.shape[0],
                                              vals.shape[1], _stream(vals)), "argmax_rows")


def sample_rows(out_idx, logits, top_k=0, top_p=1.0, temperature=1.0, seed=0, offset=0):
    """Top-k / top-p / temperature sampling of each row of logits[B, V] on the
    device, with the reference's rules (src/models/qwen2/model.cpp:60-137)."""
    _same_device(out_idx, logits)
    _arg(logits.dim() == 2, "logits must be 2D [rows, vocab]")
    _arg(out_idx.numel() == logits.shape[0] and out_idx.dtype == torch.int64, "out_idx must be int64 [rows]")
    _contig("tensors must be contiguous", out_idx, logits)
    with torch.cuda.device(logits.device):
        _lib.check(_lib.lib().wgb_sample_rows(_ptr(out_idx), _ptr(logits), _dt(logits), logits.shape[0],
                                              logits.shape[1], int(top_k), float(top_p), float(temperature),
                                              int(seed) & (2**64 - 1), int(offset) & (2**64 - 1),
                                              _stream(logits)), "sample_rows")


def embedding(out, index, weight):
    """src/ops/embedding/op.cpp:15-66."""
    _same_device(out, index, weight)
    _arg(index.dim() == 1, "index must be a 1D tensor")
    _arg(weight.dim() == 2, "weight must be a 2D tensor")
    _arg(out.dim() == 2, "out must be a 2D tensor")
    _arg(index.numel() == out.shape[0], "index must have the same number of elements as the first dimension of out")
    _arg(weight.shape[1] == out.shape[1], "weight must have the same number of rows as the second dimension of out")
    _arg(index.dtype == torch.int64, "index must be a 64-bit integer tensor")
    _arg(weight.dtype == out.dtype, "weight and out must have the same data type")
    _contig("index, weight and out must be contiguous", index, weight, out)
    with torch.cuda.device(out.device):
        _lib.check(_lib.lib().wgb_embedding(_ptr(out), _ptr(index), _ptr(weight), _dt(out), index.numel(),
                                            weight.shape[1], weight.shape[0], _stream(out)), "embedding")


def linear(out, in_, weight, bias=None):
    """src/ops/linear/op.cpp:16-73. Y = X W^T (+ b)."""
    _same_device(out, in_, weight)
    if bias is not None:
        _same_device(out, bias)
        _arg(bias.dim() == 1, "bias must be a 1D tensor")
        _arg(bias.shape[0] == out.shape[1], "N dim of bias and out must be the same")
        _arg(out.dtype == bias.dtype, "bias must have the same data type as out")
    _arg(out.dim() == 2, "out must be a 2D tensor")
    _arg(in_.dim() == 2, "in must be a 2D tensor")
    _arg(weight.dim() == 2, "weight must be a 2D tensor")
    _arg(out.shape[0] == in_.shape[0], "M dim of out and in must be the same")
    _arg(out.shape[1] == weight.shape[0], "N dim of out and weight must be the same")
    _arg(in_.shape[1] == weight.shape[1], "K dim of inin and weight must be the same")
    _arg(out.dtype == in_.dtype == weight.dtype, "out, in and weight must have the same data type")
    _contig("out, in, weight and bias must be contiguous", out, in_, weight, *([bias] if bias is not None else []))
    with torch.cuda.device(out.device):
        _lib.check(_lib.lib().wgb_linear(_ptr(out), _ptr(in_), _ptr(weight), _ptr(bias), _dt(out), out.shape[0],
                                         out.shape[1], in_.shape[1], _stream(out)), "linear")


def rms_norm(out, in_, weight, eps):
    """src/ops/rms_norm/op.cpp:14-56."""
    _same_device(out, in_, weight)
    _arg(out.dim() == 2, "out must be 2d")
    _arg(in_.dim() == 2, "in must be 2d")
    _arg(weight.dim() == 1, "weight must be 1d")
    _arg(out.shape == in_.shape, "out's shape must be same as in's shape")
    _arg(weight.shape[0] == out.shape[1], "weight and out must have equal N")
    _arg(out.dtype == in_.dtype == weight.dtype, "tensors must have the same dtype")
    _contig("tensors must be contiguous", out, in_, weight)
    with torch.cuda.device(out.device):
        _lib.check(_lib.lib().wgb_rms_norm(_ptr(out), _ptr(in_), _ptr(weight), _dt(out), out.shape[0], out.shape[1],
                                           C.c_float(eps), _stream(out)), "rms_norm")


def rope(out, in_, pos_ids, theta):
    """src/ops/rope/op.cpp:15-72."""
    _same_device(out, in_, pos_ids)
    if out.shape != in_.shape:
        raise ValueError("Shapes mismatch")
    if out.dtype != in_.dtype:
        raise ValueError("Datatypes mismatch")
    _contig("RoPE: all tensors must be contiguous.", out, in_, pos_ids)
    _arg(out.dim() == 3, "RoPE: out must be 3D [seqlen, nhead, d].")
    _arg(pos_ids.dim() == 1, "RoPE: pos_ids must be 1D [seqlen].")
    _arg(pos_ids.dtype == torch.int64, "RoPE: pos_ids must be int64.")
    _arg(theta > 0.0, "RoPE: theta must be positive.")
    seqlen, nhead, d = out.shape
    _arg(d % 2 == 0, "RoPE: head_dim must be even.")
    _arg(pos_ids.shape[0] == seqlen, "RoPE: pos_ids shape must match seqlen.")
    with torch.cuda.device(out.device):
        _lib.check(_lib.lib().wgb_rope(_ptr(out), _ptr(in_), _ptr(pos_ids), _dt(out), seqlen, nhead, d,
                                       C.c_float(theta), _stream(out)), "rope")


def self_attention(attn_val, q, k, v, scale):
    """src/ops/self_attention/op.cpp:16-80. q [S,nh,d], k [L,nkvh,d], v [L,nkvh,dv]."""
    _same_device(attn_val, q, k, v)
    if not (attn_val.dtype == q.dtype == k.dtype == v.dtype):
        raise ValueError("Datatypes mismatch")
    _arg(attn_val.dim() == 3 and q.dim() == 3 and k.dim() == 3 and v.dim() == 3,
         "self_attention: all tensors must be 3D")
    _arg(attn_val.shape[0] == q.shape[0], "self_attention: seqlen of attn_val and q must match")
    _arg(attn_val.shape[1] == q.shape[1], "self_attention: nhead of attn_val and q must match")
    _arg(q.shape[2] == k.shape[2], "self_attention: d of q and k must match")
    _arg(attn_val.shape[2] == v.shape[2], "self_attention: dv of attn_val and v must match")
    _arg(k.shape[0] == v.shape[0] and k.shape[1] == v.shape[1],
         "self_attention: total_len and nkvhead of k and v must match")
    _arg(q.shape[1] % k.shape[1] == 0, "self_attention: nhead must be divisible by nkvhead (GQA)")
    _contig("self_attention: all tensors must be contiguous", attn_val, q, k, v)
    S, nh, d = q.shape
    L, nkvh, dv = v.shape
    with torch.cuda.device(q.device):
        _lib.check(_lib.lib().wgb_self_attention(_ptr(attn_val), _ptr(q), _ptr(k), _ptr(v), _dt(q), S, nh, nkvh, d,
                                                 dv, L, C.c_float(scale), _stream(q)), "self_attention")


def swiglu(out, gate, up):
    """src/ops/swiglu/op.cpp:15-42."""
    _same_device(out, gate, up)
    if not (out.shape == gate.shape == up.shape):
        raise ValueError("Shapes mismatch")
    if not (out.dtype == gate.dtype == up.dtype):
        raise ValueError("Datatypes mismatch")
    _arg(out.dim() == 2, "out must be a 2D tensor")
    _contig("out, gate and up must be contiguous", out, gate, up)
    with torch.cuda.device(out.device):
        _lib.check(_lib.lib().wgb_swiglu(_ptr(out), _ptr(gate), _ptr(up), _dt(out), out.numel(), _stream(out)),
                   "swiglu")


def device_error(device=None):
    """(code, value) of the first bad value a kernel recorded since the last
    call (code 1 = embedding index out of range); clears it."""
    code = C.c_int64(0)
    val = C.c_int64(0)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().wgb_device_error(C.byref(code), C.byref(val),
                                               C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)),
                   "device_error")
    return code.value, val.value
