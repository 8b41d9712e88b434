"""The C-ABI library loads and exports every entry point include/*.h declares;
argument checks fail with a status before any device work; the product path
has no CPU fallback. Runs without a GPU."""
import ctypes as C
import os
import re

import numpy as np
import pytest
import torch

from wginfer_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    names = set()
    for h in ("wginfer_b200.h",):
        src = open(os.path.join(ROOT, "include", h)).read()
        names |= set(re.findall(r"__export[^;(]*?\b(wgb_\w+)\s*\(", src, re.S))
    return names


def test_library_loads():
    assert _lib.lib().wgb_version() >= 1


def test_every_declared_symbol_is_exported():
    names = declared()
    assert len(names) > 20
    raw = C.CDLL(_lib.LIB_PATH)
    for n in sorted(names):
        assert hasattr(raw, n), f"{n} declared in include/wginfer_b200.h but not exported"


def test_bindings_cover_header():
    assert declared() == set(_lib.SIGNATURES), set(_lib.SIGNATURES) ^ declared()


def test_status_strings():
    l = _lib.lib()
    assert l.wgb_status_string(0) == b"ok"
    assert l.wgb_status_string(1) == b"invalid argument"


def test_numerics_mode_per_thread():
    import threading
    _lib.set_numerics(_lib.NUMERICS_REFERENCE)
    seen = []
    t = threading.Thread(target=lambda: seen.append(_lib.get_numerics()))
    t.start()
    t.join()
    assert seen == [_lib.NUMERICS_FAST] and _lib.get_numerics() == _lib.NUMERICS_REFERENCE
    _lib.set_numerics(_lib.NUMERICS_FAST)
    assert _lib.lib().wgb_set_numerics(7) == 1


@pytest.mark.parametrize("call", [
    lambda l: l.wgb_add(None, None, None, 15, 10, None),
    lambda l: l.wgb_swiglu(None, None, None, 15, 10, None),
    lambda l: l.wgb_linear(None, None, None, None, 15, 1, 1, 1, None),
    lambda l: l.wgb_rms_norm(None, None, None, 15, 1, 4, C.c_float(1e-6), None),
    lambda l: l.wgb_rope(None, None, None, 15, 1, 1, 4, C.c_float(1e4), None),
    lambda l: l.wgb_self_attention(None, None, None, None, 15, 1, 2, 1, 4, 4, 1, C.c_float(1.0), None),
    lambda l: l.wgb_argmax(None, None, None, 15, 4, None),
    lambda l: l.wgb_embedding(None, None, None, 15, 1, 4, 8, None),
])
def test_null_pointers_rejected(call):
    assert call(_lib.lib()) == 1
    assert b"null" in _lib.lib().wgb_last_error()


def test_bad_shapes_rejected_before_device_work():
    l = _lib.lib()
    p = C.c_void_p(16)  # never dereferenced: the checks fail first
    assert l.wgb_rope(p, p, p, 15, 1, 1, 3, C.c_float(1e4), None) == 1           # odd head_dim
    assert l.wgb_rope(p, p, p, 15, 1, 1, 4, C.c_float(-1.0), None) == 1          # theta <= 0
    assert l.wgb_self_attention(p, p, p, p, 15, 1, 3, 2, 4, 4, 1, C.c_float(1.0), None) == 1  # nh % nkvh
    assert l.wgb_add(p, p, p, 6, 4, None) == 2                                    # int64 is not a float dtype
    _lib.set_numerics(_lib.NUMERICS_REFERENCE)  # long caches need score scratch there; none given
    try:
        assert l.wgb_self_attention_ex(p, p, p, p, 15, 1, 12, 2, 128, 128, 12000, C.c_float(1.0), None, 0, None) == 1
    finally:
        _lib.set_numerics(_lib.NUMERICS_FAST)
    assert l.wgb_self_attention(p, p, p, p, 15, 1, 12, 2, 512, 512, 8, C.c_float(1.0), None) == 1  # dims too large


def test_zero_sizes_are_noops():
    l = _lib.lib()
    assert l.wgb_add(None, None, None, 15, 0, None) == 0
    assert l.wgb_linear(None, None, None, None, 15, 0, 5, 5, None) == 0
    assert l.wgb_rms_norm(None, None, None, 15, 0, 4, C.c_float(1e-6), None) == 0


def test_no_cpu_fallback():
    from wginfer_b200 import ops
    a = torch.zeros(4)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.add(a.clone(), a, a)
    with pytest.raises(RuntimeError):
        ops.linear(torch.zeros(1, 2), torch.zeros(1, 3), torch.zeros(2, 3))


_STUB = r"""
#include <stddef.h>
#include <stdint.h>
/* stands in for the library's entry point: echoes its arguments */
int wgb_qwen2_infer(void *m, const int64_t *ids, size_t n, int top_k, float top_p, float t, int64_t *next) {
    *next = ids[n - 1] * 1000003 + (int64_t)n * 7 + top_k * 11 + (int64_t)(top_p * 64) + (int64_t)(t * 4096);
    return m == (void *)0x10 ? 0 : 3;
}
"""


def test_infer_one_token_path_marshals_like_the_array_path(tmp_path):
    """Qwen2.infer passes a one-token call through reused ctypes buffers; the
    arguments the entry point sees (and the returned token) match those of
    the numpy-array path, for every int64 id."""
    import subprocess
    from wginfer_b200 import qwen2 as Q
    src, so = tmp_path / "stub.c", tmp_path / "libstub.so"
    src.write_text(_STUB)
    subprocess.run(["gcc", "-shared", "-fPIC", "-O2", "-o", str(so), str(src)], check=True)
    stub = C.CDLL(str(so))
    res, args = _lib.SIGNATURES["wgb_qwen2_infer"]
    stub.wgb_qwen2_infer.restype, stub.wgb_qwen2_infer.argtypes = res, args
    m = Q.Qwen2.__new__(Q.Qwen2)
    m._l, m.h = stub, C.c_void_p(0x10)
    m._init_call_buffers()
    for tok in (0, 7, 151935, -3, (1 << 62) + 5, -(1 << 63), (1 << 63) - 1):
        for kw in ({}, {"top_k": 3, "top_p": 0.5, "temperature": 0.25}):
            want = m.infer(np.array([tok], np.int64), **kw)  # the array path
            assert m.infer([tok], **kw) == want
            assert m.infer((tok,), **kw) == want
    assert m.infer([1, 2, 3]) == m.infer(np.array([1, 2, 3]))
    with pytest.raises(OverflowError):
        m.infer([1 << 63])
    m.h = C.c_void_p(0x20)  # a failing status still raises
    with pytest.raises(RuntimeError):
        m.infer([5])
