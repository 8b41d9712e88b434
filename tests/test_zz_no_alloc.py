"""wgb_self_attention_noalloc: the attention entry point for callers that
cannot allocate device memory (code inside an allocator or memory-pool
callback, runtimes that own all device memory, threads that must not block in
the driver). It keeps its scratch in a fixed device array inside the library.
The scratch is used by REFERENCE numerics on caches longer than shared memory
holds (one score per key, past 11000 keys), so every check runs there:

* bit-identical to the oracle (the reference CPU attention restated) and to
  the allocating entry points, on two calls in a row with different inputs
  (the shared array keeps the previous call's contents);
* in a fresh process, called before any allocating entry point, it leaves the
  device's free memory unchanged;
* sizes whose scratch exceeds the array are rejected.

Collected last so a failure here leaves every other test already run."""
import ctypes as C
import subprocess
import sys

import numpy as np
import pytest
import torch

from wginfer_b200 import _lib

pytestmark = pytest.mark.gpu


def _p(t):
    return C.c_void_p(t.data_ptr())


def _inputs(seed, S, L, nh, nkvh, d):
    g = torch.Generator("cpu").manual_seed(seed)
    mk = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16).cuda()
    return mk(S, nh, d), mk(L, nkvh, d), mk(L, nkvh, d)


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("S,L", [(1, 12000), (2, 16000), (4, 12500)])
def test_noalloc_matches_oracle_and_allocating_entry(oracle, cuda, S, L):
    from wginfer_b200 import numerics
    l = _lib.lib()
    nh, nkvh, d = 12, 2, 128
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    scale = 1.0 / float(np.sqrt(d))
    with numerics("reference"):
        assert l.wgb_self_attention_workspace_size(S, nh, nkvh, d, d, L) > 0  # the path really uses scratch
        for call in range(2):  # two calls in a row, different data each time
            q, k, v = _inputs(100 * call + S + L, S, L, nh, nkvh, d)
            got = torch.full_like(q, float("nan"))
            assert l.wgb_self_attention_noalloc(_p(got), _p(q), _p(k), _p(v), 15, S, nh, nkvh, d, d, L,
                                                C.c_float(scale), st) == 0
            alloc = torch.full_like(q, float("nan"))
            assert l.wgb_self_attention(_p(alloc), _p(q), _p(k), _p(v), 15, S, nh, nkvh, d, d, L,
                                        C.c_float(scale), st) == 0
            torch.cuda.synchronize()
            want = np.zeros((S, nh, d), np.uint16)
            oracle.self_attention(want, _bits(q), _bits(k), _bits(v), scale, 15)
            assert np.array_equal(_bits(got), want)
            assert np.array_equal(_bits(alloc), want)


_FRESH = r"""
import ctypes as C, sys, torch
sys.path.insert(0, %r)
from wginfer_b200 import _lib, numerics
l = _lib.lib()
nh, nkvh, d = 12, 2, 128
st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
def run(S, L):
    g = torch.Generator("cpu").manual_seed(S * L)
    q = torch.randn(S, nh, d, generator=g).to(torch.bfloat16).cuda()
    k = torch.randn(L, nkvh, d, generator=g).to(torch.bfloat16).cuda()
    out = torch.empty_like(q)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    rc = l.wgb_self_attention_noalloc(C.c_void_p(out.data_ptr()), C.c_void_p(q.data_ptr()),
                                      C.c_void_p(k.data_ptr()), C.c_void_p(k.data_ptr()), 15, S, nh, nkvh, d, d,
                                      L, C.c_float(0.088), st)
    torch.cuda.synchronize()
    return rc, free0 - torch.cuda.mem_get_info()[0], l.wgb_self_attention_workspace_size(S, nh, nkvh, d, d, L)
with numerics("reference"):
    # first call: loads the library's device code (and with it the array) on this device
    rc, _, need0 = run(1, 12000)
    assert rc == 0 and need0 > 0
    # larger scratch needs than the first call's: an allocation here would show
    for S, L in ((2, 20000), (4, 20000)):
        rc, used, need = run(S, L)
        assert rc == 0 and need > need0 and used == 0, (S, L, rc, used, need)
print("noalloc-fresh-ok")
"""


def test_noalloc_allocates_nothing_in_fresh_process(cuda):
    import os
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _FRESH % root], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "noalloc-fresh-ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    from wginfer_b200 import numerics
    l = _lib.lib()
    cap = l.wgb_self_attention_noalloc_max_scratch()
    assert cap == 4 << 20
    S, nh, nkvh, d = 1, 12, 2, 128
    with numerics("reference"):  # reference numerics keep one score per key in scratch for long caches
        L = next(L for L in (50000, 100000, 200000) if l.wgb_self_attention_workspace_size(S, nh, nkvh, d, d, L) > cap)
        q, k, v = _inputs(7, S, L, nh, nkvh, d)
        out = torch.empty_like(q)
        st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = l.wgb_self_attention_noalloc(_p(out), _p(q), _p(k), _p(v), 15, S, nh, nkvh, d, d, L,
                                          C.c_float(0.088), st)
    assert rc == 4 and b"static array" in l.wgb_last_error()
