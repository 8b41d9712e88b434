"""Parity of every op with the CPU oracle on the seeded cases, through the
C-ABI. REFERENCE numerics must be bit-identical (f16 within one f16 ulp:
the reference's CPU f16 conversion truncates where the device rounds to
nearest); FAST numerics within the tolerances the backend promises:
1e-5 relative for f32, 2e-2 relative for bf16/f16 (atol 1e-2), exact for
add, embedding and argmax."""
import numpy as np
import pytest
import torch

from tests.golden import cases as CS
from wginfer_b200 import numerics, ops

pytestmark = pytest.mark.gpu

EXACT_OPS = {"add", "embedding", "argmax"}
# f32 RoPE evaluates sin/cos/pow: REFERENCE numerics round those correctly
# (double evaluation), while glibc's f32 sinf/cosf are off by one ulp on about
# 1.3% of RoPE angles. The output then differs by about one ulp of the terms it
# is formed from (a*cos - b*sin can cancel, so this is an absolute bound, not a
# relative one). bf16 outputs absorb these differences and stay bit-identical.
# exp (swiglu, the attention softmax) is the C library's expf restated
# (libm_expf.cuh), so those ops are bit-identical at f32 too.
TRANSCENDENTAL_ATOL = {"rope": 1e-6}


def as_f32(a):
    if a.dtype == np.float32 or a.dtype == np.int64:
        return a.astype(np.float64)
    return (a.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def f16_f64(a):
    return a.view(np.float16).astype(np.float64)


@pytest.fixture(scope="module")
def gpu(cuda):
    from tests.gpu_runner import Gpu
    return Gpu()


@pytest.mark.parametrize("mode", ["reference", "fast"])
@pytest.mark.parametrize("cid", range(len(CS.OP_CASES)))
def test_op_parity(oracle, gpu, mode, cid):
    case = CS.OP_CASES[cid]
    ins = CS.inputs(case)
    want = CS.run_case(oracle, case, ins)
    with numerics(mode):
        got = CS.run_case(gpu, case, ins)
    torch.cuda.synchronize()
    for g, w in zip(got, want):
        if case["dtype"] == "f16" and case["op"] not in ("embedding",):
            if case["op"] == "argmax":
                assert np.array_equal(g, w)
                continue
            # device rounds to nearest, the reference's CPU f16 conversion truncates
            np.testing.assert_allclose(f16_f64(g), f16_f64(w), rtol=2e-3 if mode == "reference" else 2e-2, atol=1e-3)
            continue
        if mode == "reference" and case["dtype"] == "f32" and case["op"] in TRANSCENDENTAL_ATOL:
            diff = np.abs(as_f32(g) - as_f32(w)).max()
            assert diff <= TRANSCENDENTAL_ATOL[case["op"]], f"{case}: max diff {diff}"
        elif mode == "reference" or case["op"] in EXACT_OPS:
            assert np.array_equal(g, w), f"{case}: max diff {np.abs(as_f32(g) - as_f32(w)).max()}"
        elif case["dtype"] == "f32":
            np.testing.assert_allclose(as_f32(g), as_f32(w), rtol=1e-5, atol=1e-5)
        else:
            np.testing.assert_allclose(as_f32(g), as_f32(w), rtol=2e-2, atol=1e-2)


def _bf16(shape, seed, std=1.0, mean=0.0):
    g = torch.Generator("cpu").manual_seed(seed)
    return (torch.randn(shape, generator=g) * std + mean).to(torch.bfloat16).cuda()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("n", [(1 << 25) + 3, 64 << 20])
def test_add_swiglu_large_vs_torch(cuda, dtype, n):
    g = torch.Generator("cpu").manual_seed(n % 1000)
    a = torch.randn(n, generator=g).to(dtype).cuda()
    b = torch.randn(n, generator=g).to(dtype).cuda()
    c = torch.empty_like(a)
    ops.add(c, a, b)
    assert torch.equal(c, (a.float() + b.float()).to(dtype))
    o = torch.empty_like(a).view(1, -1)
    ops.swiglu(o, a.view(1, -1), b.view(1, -1))
    ref = (b.float() * a.float() / (1 + torch.exp(-a.float()))).to(dtype)
    torch.testing.assert_close(o.view(-1).float(), ref.float(), rtol=2e-2 if dtype != torch.float32 else 1e-5,
                               atol=1e-2 if dtype != torch.float32 else 1e-5)


@pytest.mark.parametrize("N", [1536, 4096, 8192, 1000])
def test_rms_norm_large_vs_torch(cuda, N):
    M = (64 << 20) // (2 * N)
    x = _bf16((M, N), N)
    w = _bf16((N,), N + 1, 0.1, 1.0)
    out = torch.empty_like(x)
    ops.rms_norm(out, x, w, 1e-6)
    xf = x.float()
    ref = (xf * w.float() * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
    torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=1e-2)


@pytest.mark.parametrize("B", [1, 3, 64, 256])
def test_argmax_rows_first_index(oracle, cuda, B):
    V = 151936
    vals = _bf16((B, V), B)
    # plant ties: copy each row's max to an earlier and a later position
    am = vals.float().argmax(-1)
    for r in range(B):
        vals[r, 7] = vals[r, am[r]]
        vals[r, V - 1] = vals[r, am[r]]
    idx = torch.empty(B, dtype=torch.int64, device="cuda")
    val = torch.empty(B, dtype=torch.bfloat16, device="cuda")
    ops.argmax_rows(idx, val, vals)
    host = vals.cpu().view(torch.int16).numpy().view(np.uint16)
    vh = val.cpu().view(torch.int16).numpy().view(np.uint16)
    for r in range(B):
        i, v = oracle.argmax(np.ascontiguousarray(host[r]), 15)
        assert idx[r].item() == i and vh[r] == v


def test_argmax_nan_semantics(oracle, cuda):
    v = torch.tensor([float("nan"), 1.0, 3.0, 2.0], device="cuda")
    idx = torch.zeros(1, dtype=torch.int64, device="cuda")
    val = torch.zeros(1, device="cuda")
    ops.argmax(idx, val, v)
    assert idx.item() == 0  # the sequential scan keeps a NaN at index 0
    v = torch.tensor([1.0, float("nan"), 3.0, 3.0, -0.0], device="cuda")
    ops.argmax(idx, val, v)
    assert idx.item() == 2 and val.item() == 3.0


@pytest.mark.parametrize("reps", [1, 4])
@pytest.mark.parametrize("n", [4096, 4093])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
def test_argmax_rows_special_values(oracle, cuda, dt, n, reps):
    """Rows with NaNs, signed-zero maxima, -inf rows, all-NaN rows and ties
    inside one 16-byte vector, against the oracle's sequential scan
    (argmax_cpu.cpp:26-47). 7 rows take the few-rows launch (8-CTA clusters
    of 256 threads), 28 rows the many-rows one (512-thread CTAs); a width
    of 4093 takes the element-wise path (rows not 16-byte aligned)."""
    g = torch.Generator("cpu").manual_seed(3)
    rows = []
    r = -torch.rand(n, generator=g) - 1.0; r[100] = 0.0; r[50] = -0.0; rows.append(r)  # -0 first, then +0
    r = torch.randn(n, generator=g); r[0:8] = float("nan"); r[9] = 9.0; r[10] = 9.0; rows.append(r)  # tie in a vector
    r = torch.full((n,), float("-inf")); rows.append(r)  # nothing beats -inf: index 0
    r = torch.full((n,), float("nan")); r[4000] = -5.0; rows.append(r)  # the only number
    r = torch.full((n,), float("nan")); rows.append(r)  # all NaN: index 0
    r = torch.randn(n, generator=g); r[0] = float("nan"); rows.append(r)  # NaN at index 0 wins
    r = torch.randn(n, generator=g); r[17] = float("inf"); r[n - 1] = float("inf"); rows.append(r)
    vals = torch.stack(rows * reps).to(dt).cuda()
    idx = torch.empty(vals.shape[0], dtype=torch.int64, device="cuda")
    val = torch.empty(vals.shape[0], dtype=dt, device="cuda")
    ops.argmax_rows(idx, val, vals)
    code = {torch.bfloat16: 15, torch.float16: 12, torch.float32: 13}[dt]
    host = vals.cpu()
    for i in range(vals.shape[0]):
        row = host[i].numpy() if dt == torch.float32 else host[i].view(torch.int16).numpy().view(np.uint16)
        want_i, _ = oracle.argmax(np.ascontiguousarray(row), code)
        assert idx[i].item() == want_i, (i, idx[i].item(), want_i)


def test_embedding_out_of_range_is_recorded(cuda):
    w = _bf16((16, 64), 9)
    out = torch.full((3, 64), 7.0, dtype=torch.bfloat16, device="cuda")
    idx = torch.tensor([1, 16, 2], device="cuda")
    ops.device_error()  # clear
    ops.embedding(out, idx, w)
    code, value = ops.device_error()
    assert code == 1 and value == 16
    assert torch.equal(out[0], w[1]) and torch.equal(out[2], w[2]) and torch.all(out[1] == 0)
    assert ops.device_error() == (0, 0)


def test_rope_in_place_and_unaligned_views(oracle, cuda):
    x = _bf16((4 * 12 * 128 + 1,), 3)
    view = x[1:].view(4, 12, 128)  # 2-byte offset: not 16-byte aligned
    pos = torch.arange(10, 14, device="cuda")
    want = torch.empty_like(view)
    ops.rope(want, view.clone(), pos, 1e4)
    ops.rope(view, view, pos, 1e4)  # in place
    assert torch.equal(view, want)
    a, b = _bf16((1001,), 4), _bf16((1001,), 5)
    c = torch.empty(1002, dtype=torch.bfloat16, device="cuda")
    ops.add(c[1:], a, b)
    assert torch.equal(c[1:], (a.float() + b.float()).to(torch.bfloat16))


@pytest.mark.parametrize("mode", ["fast", "reference"])
def test_linear_unaligned_and_ragged(oracle, cuda, mode):
    M, N, K = 3, 50, 77
    x, w, b = _bf16((M, K), 1), _bf16((N, K), 2, 0.02), _bf16((N,), 3, 0.02)
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    with numerics(mode):
        ops.linear(out, x, w, b)
    h = lambda t: t.cpu().view(torch.int16).numpy().view(np.uint16)
    want = np.zeros((M, N), np.uint16)
    oracle.linear(want, h(x), h(w), h(b), 15)
    got = h(out)
    if mode == "reference":
        assert np.array_equal(got, want)
    else:
        np.testing.assert_allclose(as_f32(got), as_f32(want), rtol=2e-2, atol=1e-2)


# More than 8 bf16 rows take the tcgen05 GEMM (TMA-fed shared-memory ring,
# f32 accumulator in tensor memory). Shapes cover ragged M (tile of 16..128
# rows), N not a multiple of the 128-row weight tile, odd N, K below one
# 64-wide slice and K not a multiple of it (zero-filled by the copy engine).
TC_SHAPES = [(9, 128, 64), (20, 256, 1536), (64, 1536, 1536), (64, 17920, 1536), (100, 1536, 8960),
             (512, 2048, 1536), (200, 37, 104), (33, 300, 24), (1000, 96, 200), (300, 17920, 1536),
             (512, 17920, 1536)]


@pytest.mark.parametrize("M,N,K", TC_SHAPES)
@pytest.mark.parametrize("bias", [True, False])
def test_linear_tensor_core_vs_torch(cuda, M, N, K, bias):
    x = _bf16((M, K), M * 7 + K)
    w = _bf16((N, K), N * 3 + K, 0.02)
    b = _bf16((N,), N, 0.5) if bias else None
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    with numerics("fast"):
        ops.linear(out, x, w, b)
    ref = x.float() @ w.float().T
    if bias:
        ref = ref + b.float()
    torch.testing.assert_close(out.float(), ref.to(torch.bfloat16).float(), rtol=2e-2, atol=1e-2)
    assert ops.device_error() == (0, 0)


def test_linear_tensor_core_vs_oracle(oracle, cuda):
    M, N, K = 40, 260, 1536
    x, w, b = _bf16((M, K), 11), _bf16((N, K), 12, 0.02), _bf16((N,), 13, 0.02)
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    with numerics("fast"):
        ops.linear(out, x, w, b)
    h = lambda t: t.cpu().view(torch.int16).numpy().view(np.uint16)
    want = np.zeros((M, N), np.uint16)
    oracle.linear(want, h(x), h(w), h(b), 15)
    np.testing.assert_allclose(as_f32(h(out)), as_f32(want), rtol=2e-2, atol=1e-2)


def test_ops_first_use_in_fresh_process(cuda):
    """Every op works as the first library call of a process (kernel
    attributes such as shared-memory limits are set on first use, not only
    by model creation)."""
    import subprocess
    import sys
    code = (
        "import torch\n"
        "from wginfer_b200 import ops\n"
        "bf = torch.bfloat16\n"
        "for M, N, K in ((1, 2048, 1536), (4, 1536, 8960), (20, 256, 1536)):\n"
        "    x = torch.randn(M, K, device='cuda').to(bf); w = torch.randn(N, K, device='cuda').to(bf) * 0.02\n"
        "    o = torch.empty(M, N, device='cuda', dtype=bf); ops.linear(o, x, w)\n"
        "    torch.testing.assert_close(o.float(), (x.float() @ w.float().T).to(bf).float(), rtol=2e-2, atol=1e-2)\n"
        "q = torch.randn(1, 12, 128, device='cuda').to(bf); k = torch.randn(700, 2, 128, device='cuda').to(bf)\n"
        "a = torch.empty_like(q); ops.self_attention(a, q, k, k.clone(), 0.088)\n"
        "torch.cuda.synchronize(); print('ok')\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]


def _attn_ref(q, k, v, scale):
    """Causal GQA attention in fp32 torch: query i sees keys j <= i + L - S."""
    S, nh, d = q.shape
    L, nkvh, dv = v.shape
    qf, kf, vf = q.float(), k.float(), v.float()
    out = torch.empty(S, nh, dv, device=q.device)
    i = torch.arange(S, device=q.device)[:, None]
    j = torch.arange(L, device=q.device)[None, :]
    mask = j > i + (L - S)
    for h in range(nh):
        kv = h * nkvh // nh
        sc = (qf[:, h] @ kf[:, kv].T) * scale
        sc = sc.masked_fill(mask, float("-inf"))
        out[:, h] = torch.softmax(sc, -1) @ vf[:, kv]
    return out


# Prefill shapes take the tensor-core kernel (bf16/f16, head dim 64/128, at
# least 2 x SMs query rows x heads): full causal, causal behind a cached
# prefix (L > S), ragged query tiles, GQA groups of 6 and 2.
PREFILL = [(512, 512, 12, 2, 128), (100, 612, 12, 2, 128), (2048, 2048, 12, 2, 128), (333, 333, 8, 4, 64),
           (64, 1000, 16, 2, 128), (257, 300, 12, 12, 64)]


@pytest.mark.parametrize("S,L,nh,nkvh,d", PREFILL)
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_attention_prefill_vs_torch(cuda, S, L, nh, nkvh, d, dt):
    g = torch.Generator("cpu").manual_seed(S * 7 + L)
    q = torch.randn(S, nh, d, generator=g).to(dt).cuda()
    k = torch.randn(L, nkvh, d, generator=g).to(dt).cuda()
    v = torch.randn(L, nkvh, d, generator=g).to(dt).cuda()
    out = torch.full((S, nh, d), float("nan"), dtype=dt, device="cuda")
    scale = 1.0 / d ** 0.5
    with numerics("fast"):
        ops.self_attention(out, q, k, v, scale)
    torch.testing.assert_close(out.float(), _attn_ref(q, k, v, scale), rtol=2e-2, atol=1e-2)


def test_attention_workspace_contract(oracle, cuda):
    """FAST needs no workspace (the cluster folds its key slices in shared
    memory); REFERENCE keeps one score per key in the workspace once the cache
    is longer than shared memory holds. Both REFERENCE entry points are
    bit-identical to the oracle there."""
    import ctypes as C
    from wginfer_b200 import _lib
    l = _lib.lib()
    assert l.wgb_self_attention_workspace_size(1, 12, 2, 128, 128, 4096) == 0
    L = 12000
    q = _bf16((1, 12, 128), 1)
    k = _bf16((L, 2, 128), 2)
    v = _bf16((L, 2, 128), 3)
    out = torch.empty_like(q)
    p = lambda t: C.c_void_p(t.data_ptr())
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    with numerics("reference"):
        need = l.wgb_self_attention_workspace_size(1, 12, 2, 128, 128, L)
        assert need == 12 * L * 4
        rc = l.wgb_self_attention_ex(p(out), p(q), p(k), p(v), 15, 1, 12, 2, 128, 128, L, C.c_float(0.088), None, 0, st)
        assert rc == 1
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        rc = l.wgb_self_attention_ex(p(out), p(q), p(k), p(v), 15, 1, 12, 2, 128, 128, L, C.c_float(0.088), p(ws),
                                     need, st)
        assert rc == 0
        out2 = torch.empty_like(q)
        ops.self_attention(out2, q, k, v, 0.088)
    torch.cuda.synchronize()
    h = lambda t: t.cpu().view(torch.int16).numpy().view(np.uint16)
    want = np.zeros((1, 12, 128), np.uint16)
    oracle.self_attention(want, h(q), h(k), h(v), 0.088, 15)
    assert np.array_equal(h(out), want)
    assert np.array_equal(h(out2), want)


@pytest.mark.parametrize("mode", ["fast", "reference"])
@pytest.mark.parametrize("L", [1, 63, 64, 65, 700, 2304, 12000, 16000])
def test_attention_decode_lengths(oracle, cuda, mode, L):
    """Single-query decode over cache lengths around the tile size; past
    11000 keys REFERENCE keeps its scores in the global workspace."""
    q, k, v = _bf16((1, 12, 128), L), _bf16((L, 2, 128), L + 1), _bf16((L, 2, 128), L + 2)
    out = torch.empty_like(q)
    with numerics(mode):
        ops.self_attention(out, q, k, v, 1 / 128 ** 0.5)
    h = lambda t: t.cpu().view(torch.int16).numpy().view(np.uint16)
    want = np.zeros((1, 12, 128), np.uint16)
    oracle.self_attention(want, h(q), h(k), h(v), 1 / 128 ** 0.5, 15)
    if mode == "reference":
        assert np.array_equal(h(out), want)
    else:
        np.testing.assert_allclose(as_f32(h(out)), as_f32(want), rtol=2e-2, atol=1e-2)


@pytest.mark.parametrize("up", [1.0, -3.5])
def test_swiglu_f32_reference_exp_sweep(oracle, cuda, up):
    """REFERENCE swiglu at f32 over every 61st 32-bit pattern of the gate
    (70 M values: normals, subnormals, both overflow edges, inf and NaN),
    bit-identical to the oracle, whose exp is the host C library's expf."""
    bits = np.arange(0, 1 << 32, 61, dtype=np.uint64).astype(np.uint32)
    gate = bits.view(np.float32)
    upv = np.full_like(gate, up)
    want = np.zeros_like(gate)
    oracle.swiglu(want, gate, upv, 13)
    g = torch.from_numpy(gate).cuda()
    out = torch.empty_like(g)
    with numerics("reference"):
        ops.swiglu(out.view(1, -1), g.view(1, -1), torch.from_numpy(upv).cuda().view(1, -1))
    got = out.cpu().numpy()
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    bad = np.flatnonzero(~same)
    assert bad.size == 0, f"{bad.size} differ, first gate {gate[bad[0]]!r}: {got[bad[0]]!r} vs {want[bad[0]]!r}"
