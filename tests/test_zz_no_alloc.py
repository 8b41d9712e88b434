"""wgb_self_attention_noalloc: the attention entry point for callers that
cannot allocate device memory (allocator callbacks, runtimes that own all
device memory, threads that must not block in the driver). It keeps its
scratch in a fixed device array inside the library. Checked through the
C-ABI against the allocating entry point, on two calls in a row with
different inputs (the shared array keeps the previous call's contents), and
for its size limit. The scratch is used by reference numerics on caches
longer than shared memory holds (one score per key), so the comparison runs
there. Collected last so a failure here leaves every other test already
run."""
import ctypes as C

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


@pytest.mark.parametrize("S,L", [(1, 12000), (2, 16000), (4, 12500)])
def test_noalloc_matches_allocating_entry(S, L):
    from wginfer_b200 import numerics
    assert torch.cuda.is_available()
    l = _lib.lib()
    nh, nkvh, d = 12, 2, 128
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    scale = C.c_float(1.0 / np.sqrt(d))
    with numerics("reference"):
        assert l.wgb_self_attention_workspace_size(S, nh, nkvh, d, d, L) > 0  # the path really uses scratch
        for call in range(2):  # two calls in a row, different data each time
            q, k, v = _inputs(100 * call + S + L, S, L, nh, nkvh, d)
            want = torch.empty_like(q)
            got = torch.full_like(q, float("nan"))
            assert l.wgb_self_attention(_p(want), _p(q), _p(k), _p(v), 15, S, nh, nkvh, d, d, L, scale, st) == 0
            assert l.wgb_self_attention_noalloc(_p(got), _p(q), _p(k), _p(v), 15, S, nh, nkvh, d, d, L, scale,
                                                st) == 0
            torch.cuda.synchronize()
            torch.testing.assert_close(got.float(), want.float(), rtol=2e-2, atol=1e-2)


def test_noalloc_rejects_sizes_beyond_its_scratch():
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
