"""Decode benchmark of the B200 backend on the Qwen2-1.5B architecture.

Headline (`value`): greedy batch-1 decode tok/s of the full 28-layer
Qwen2-1.5B architecture in bf16 (random weights, 512-token prompt), one
request per GPU; with N GPUs every rank decodes its own request on its own
model replica (requests partitioned across GPUs, no collective on the data
path), so `value` is the whole-box tok/s and scaling is weak. A step is one
decode token: one CUDA-graph launch of the 28-layer step with the token
buffer on the device. Weights (3.1 GB) exceed L2 (126 MB), so no flush is
needed between steps.

`e2e`: the same metric through the public call a user makes
(wgb_qwen2_infer: host token in, host token out), with the 8-byte
host->device and device->host copies inside the timed region.

`value` is measured in FAST numerics (the default mode: f32 sums in the
fastest order). `reference_numerics` is the same measurement in REFERENCE
numerics, the mode whose greedy tokens are identical to the reference's
(every sum in the reference CPU backend's order; tests/test_model_gpu.py
checks the streams), on the same model in the same run.

Extra objects: `roofline` (the weight-streaming GEMV, the dominant kernel),
`cpu_baseline` (the reference's own CPU build timed on a bounded sample),
`clocks`, `op_bandwidth`, `prefill` (one GPU: the prompt's prefill on the
28-layer model, best of 3), and at the end of the line `bs64` (64 sequences
with 2048-token prompts on the one-layer model, requests split across the
GPUs: a strong-scaling workload) and `reference_numerics`.

`--impl reference` times the reference's own CPU implementation
(oracle/_ref, the full 28-layer Model) on the host cores for the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (Qwen2-1.5B arch bf16, bs1 & bs64) + per-op HBM GB/s vs peak"
SPEC_HBM_GBS = 8000.0  # B200 HBM3e specification (the measured copy peak is in MEASURED_PEAKS.json)
UNIT = "tok/s"


def load_peaks():
    try:
        p = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------- clocks
class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if len(r) > 8 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 8 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) > 8 for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ---------------------------------------------------------------- helpers
def dist_setup(n_gpus):
    """One process per GPU under torchrun (NCCL), else a single GPU."""
    from wginfer_b200 import dist as D
    return D.setup(timeout_s=300.0)


def barrier(world):
    from wginfer_b200 import dist as D
    D.barrier()


def max_over_ranks(x: float, world: int) -> float:
    from wginfer_b200 import dist as D
    return D.max_over_ranks(x)


def device_weights(cfg, seed, device):
    """Random weights drawn on the device (same distributions as
    wginfer_b200.synthetic, a device generator stream)."""
    import torch
    from wginfer_b200.synthetic import LAYER_NAMES
    g = torch.Generator(device=device).manual_seed(seed)

    def draw(shape, std, mean=0.0):
        t = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
        t.mul_(std).add_(mean)
        return t.to(cfg.dtype)

    w = {"in_embed": draw((cfg.voc, cfg.hs), 0.02)}
    shapes = cfg.shapes()
    for n in LAYER_NAMES:
        w[n] = []
    for _ in range(cfg.nlayer):
        for n in LAYER_NAMES:
            w[n].append(draw(shapes[n], 0.1, 1.0) if n.endswith("norm_w") else draw(shapes[n], 0.02))
    w["out_norm_w"] = draw((cfg.hs,), 0.1, 1.0)
    w["out_embed"] = draw((cfg.voc, cfg.hs), 0.02)
    return w


def build_model(cfg, max_batch, device_index, seed=0, keep=()):
    import torch
    from wginfer_b200.qwen2 import Qwen2
    dev = torch.device("cuda", device_index)
    w = device_weights(cfg, seed, dev)
    m = Qwen2(cfg, None, device=device_index, max_batch=max_batch)
    m.load_weights(w)
    kept = {k: w[k] for k in keep}
    del w
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()
    return m, kept


# ---------------------------------------------------------------- B200 arm
def time_decode(m, batch, K, W, world):
    import torch
    s = m.torch_stream()
    for _ in range(W):
        m.decode_step(batch)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(K):
        m.decode_step(batch)
    e1.record(s)
    e1.synchronize()
    barrier(world)
    return e0.elapsed_time(e1) / 1e3


def _time_linear(out, x, ws, K):
    """Average device time (s) of one ops.linear launch: K launches cycling
    through `ws` are captured once in a CUDA graph (so host launch overhead
    leaves no gaps between them) and the replay is timed with CUDA events on
    the capturing stream."""
    import torch
    from wginfer_b200 import numerics, ops
    s = torch.cuda.Stream()
    with numerics("fast"):
        with torch.cuda.stream(s):
            for i in range(3):
                ops.linear(out, x, ws[i % len(ws)])
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(K):
                ops.linear(out, x, ws[i % len(ws)])
    with torch.cuda.stream(s):
        g.replay()  # warm
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        g.replay()
        e1.record(s)
    e1.synchronize()
    del g
    return e0.elapsed_time(e1) / 1e3 / K


def gemv_roofline(w_out, cfg, peak, K=24):
    """Roofline of the dominant decode kernel: the weight-streaming GEMV of the
    gate/up projection ([1,1536] x [17920,1536]^T, 55 MB of bf16 weights, 28%
    of a decode step's kernel time), timed live with CUDA events over eight
    weight copies (440 MB, so every launch streams from HBM, not L2). The
    lm_head GEMV ([1,1536] x [151936,1536]^T) is reported beside it."""
    import torch
    dev, dt = w_out.device, w_out.dtype
    g = torch.Generator(device=dev).manual_seed(7)
    n_gu, k = 2 * cfg.di, cfg.hs
    ws = [(torch.randn(n_gu, k, device=dev, generator=g) * 0.02).to(dt) for _ in range(8)]
    x = torch.randn(1, k, device=dev, generator=g).to(dt)
    out = torch.empty(1, n_gu, device=dev, dtype=dt)
    dt_gu = _time_linear(out, x, ws, K)
    del ws
    nbytes = (n_gu * k + k + n_gu) * w_out.element_size()
    traffic = None
    try:
        prof = json.load(open(os.path.join(ROOT, "profiles", "gemv_traffic.json")))
        traffic = prof.get("gate_up", {}).get("dram_bytes_per_launch")
        traffic_lm = prof.get("lm_head", {}).get("dram_bytes_per_launch")
    except Exception:
        traffic_lm = None
    xl = torch.randn(1, cfg.hs, device=dev, generator=g).to(dt)
    ol = torch.empty(1, cfg.voc, device=dev, dtype=dt)
    dt_lm = _time_linear(ol, xl, [w_out], 20)
    nbytes_lm = (cfg.voc * cfg.hs + cfg.hs + cfg.voc) * w_out.element_size()
    achieved = nbytes / dt_gu / 1e9
    return {"kernel": "decode_gemv_kernel (gate/up projection [1,1536]x[17920,1536]^T, bf16)", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
            "traffic": traffic, "algorithmic_bytes": nbytes, "us_per_launch": round(dt_gu * 1e6, 2),
            "lm_head": {"achieved": round(nbytes_lm / dt_lm / 1e9, 1), "frac": round(nbytes_lm / dt_lm / 1e9 / peak, 4),
                        "algorithmic_bytes": nbytes_lm, "us_per_launch": round(dt_lm * 1e6, 2),
                        "traffic": traffic_lm}}


def _graph_time(fn, reps):
    """Average device time (s) of fn(i) over `reps` calls captured in one
    CUDA graph, timed with CUDA events around a replay (after a warm replay)."""
    import torch
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for i in range(2):
            fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(reps):
            fn(i)
    with torch.cuda.stream(s):
        g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        g.replay()
        e1.record(s)
    e1.synchronize()
    del g
    return e0.elapsed_time(e1) / 1e3 / reps


def op_sweep(peak, quick=False):
    """Bandwidth sweep of the elementwise and reduction ops (add, swiglu on
    flat tensors of 1M..1G elements; rms_norm rows of 1536/4096/8192; argmax
    over [B, 151936]), bf16 and f32, inputs ~N(0,1). Each case cycles through
    enough copies of its operands that every launch streams more than L2
    (126 MB) from HBM; achieved = algorithmic bytes / device time."""
    import torch
    from wginfer_b200 import numerics, ops
    gen = torch.Generator(device="cuda").manual_seed(5)
    L2_SPAN = 256 << 20
    out = []

    def copies(bytes_per_iter, budget=6 << 30):
        return int(max(1, min(64, -(-L2_SPAN // bytes_per_iter), budget // bytes_per_iter)))

    def record(op, dtype, shape, nbytes, t):
        gbs = nbytes / t / 1e9
        out.append({"op": op, "dtype": dtype, "shape": shape, "bytes": nbytes, "us": round(t * 1e6, 2),
                    "gbs": round(gbs, 1), "frac": round(gbs / peak, 3), "frac_spec": round(gbs / SPEC_HBM_GBS, 3)})

    flat = [1 << 20, 1 << 24, 1 << 28] + ([] if quick else [1 << 30])
    with numerics("fast"):
        for tdt, name in ((torch.bfloat16, "bf16"), (torch.float32, "f32")):
            es = torch.tensor([], dtype=tdt).element_size()
            for n in flat:
                per = 3 * n * es
                if per > (16 << 30):
                    continue
                nc = copies(per)
                a = [torch.randn(n, device="cuda", generator=gen).to(tdt) for _ in range(nc)]
                b = [torch.randn(n, device="cuda", generator=gen).to(tdt) for _ in range(nc)]
                c = [torch.empty(n, device="cuda", dtype=tdt) for _ in range(nc)]
                reps = max(3, min(100, (2 << 30) // per))
                record("add", name, [n], per, _graph_time(lambda i: ops.add(c[i % nc], a[i % nc], b[i % nc]), reps))
                record("swiglu", name, [1, n], per, _graph_time(
                    lambda i: ops.swiglu(c[i % nc].view(1, -1), a[i % nc].view(1, -1), b[i % nc].view(1, -1)), reps))
                del a, b, c
            for h in (1536, 4096, 8192):
                rows = (256 << 20) // (h * es)
                per = 2 * rows * h * es + h * es
                nc = copies(per)
                x = [torch.randn(rows, h, device="cuda", generator=gen).to(tdt) for _ in range(nc)]
                y = [torch.empty(rows, h, device="cuda", dtype=tdt) for _ in range(nc)]
                w = (torch.randn(h, device="cuda", generator=gen) * 0.1 + 1).to(tdt)
                record("rms_norm", name, [rows, h], per,
                       _graph_time(lambda i: ops.rms_norm(y[i % nc], x[i % nc], w, 1e-6), 20))
                del x, y
            for B in (1, 16, 64, 256):
                V = 151936
                per = B * V * es + B * (8 + es)
                nc = copies(per)
                v = [torch.randn(B, V, device="cuda", generator=gen).to(tdt) for _ in range(nc)]
                idx = torch.empty(B, dtype=torch.int64, device="cuda")
                val = torch.empty(B, dtype=tdt, device="cuda")
                record("argmax", name, [B, V], per,
                       _graph_time(lambda i: ops.argmax_rows(idx, val, v[i % nc]), max(3, min(100, (2 << 30) // per))))
                del v
    torch.cuda.empty_cache()
    big = [r for r in out if r["bytes"] >= (64 << 20)]
    return {"unit": "GB/s", "peak": peak, "spec_peak": SPEC_HBM_GBS, "cases": out,
            "min_frac_at_64MB_or_more": round(min(r["frac"] for r in big), 3) if big else None,
            "min_frac_spec_at_64MB_or_more": round(min(r["frac_spec"] for r in big), 3) if big else None}


def op_probe(op: str, reps: int = 3):
    """A few launches of one swept op at a size of 64 MB or more (bf16), for
    an ncu capture of its DRAM bytes: add and swiglu on 2^25 elements,
    rms_norm on [43690, 1536], argmax over [256, 151936]."""
    import torch
    from wginfer_b200 import numerics, ops
    g = torch.Generator(device="cuda").manual_seed(5)
    bf = torch.bfloat16
    with numerics("fast"):
        if op in ("add", "swiglu"):
            n = 1 << 25
            a, b = torch.randn(n, device="cuda", generator=g).to(bf), torch.randn(n, device="cuda", generator=g).to(bf)
            c = torch.empty_like(a)
            fn = (lambda: ops.add(c, a, b)) if op == "add" else (
                lambda: ops.swiglu(c.view(1, -1), a.view(1, -1), b.view(1, -1)))
        elif op == "rms_norm":
            x = torch.randn(43690, 1536, device="cuda", generator=g).to(bf)
            w = (torch.randn(1536, device="cuda", generator=g) * 0.1 + 1).to(bf)
            y = torch.empty_like(x)
            fn = lambda: ops.rms_norm(y, x, w, 1e-6)
        else:
            v = torch.randn(256, 151936, device="cuda", generator=g).to(bf)
            idx = torch.empty(256, dtype=torch.int64, device="cuda")
            val = torch.empty(256, dtype=bf, device="cuda")
            fn = lambda: ops.argmax_rows(idx, val, v)
        for _ in range(reps):
            fn()
    torch.cuda.synchronize()
    print(json.dumps({"op_probe": op, "launches": reps}))


def decode_config(args, world):
    """The workload the B200 arm reports (the metric is quoted on it)."""
    return {"workload": "Qwen2-1.5B arch (28 layers, hidden 1536, 12/2 heads x 128, MLP 8960, vocab "
                        "151936), greedy decode, batch 1 per GPU, prompt %d" % args.prompt,
            "global_batch": world, "seq_len": args.prompt + args.steps, "parallelism": f"replicas x{world}",
            "numerics": args.numerics, "l2": "weights 3.1 GB > L2; no flush needed"}


def time_e2e(m, K, W, world):
    """K decode steps through Qwen2.infer (wgb_qwen2_infer: the token copied
    host->device and the next token device->host every step), device-timed."""
    import torch
    s = m.torch_stream()
    tok = m.tokens(1)[0]
    for _ in range(W):
        tok = m.infer([tok])
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(K):
        tok = m.infer([tok])
    e1.record(s)
    e1.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1) / 1e3, world)


def reference_numerics_leg(m, args, world, rank, bytes_per_token, peak):
    """The same decode in REFERENCE numerics (token-identical to the
    reference) on the same model: fresh cache, the same prompt, K graph
    steps device-timed, then K steps end to end."""
    from wginfer_b200 import numerics
    from wginfer_b200.synthetic import prompt_ids
    K, W = args.steps, args.warmup
    with numerics("reference"):
        m.reset_cache()
        m.prefill(0, prompt_ids(args.prompt, m.cfg.voc, seed=rank).numpy())
        t = max_over_ranks(time_decode(m, 1, K, W, world), world)
        te = time_e2e(m, K, W, world)
    value = world * K / t
    return {"value": round(value, 2), "unit": UNIT, "ms_per_step": round(t / K * 1e3, 4),
            "weight_stream_roofline_frac": round(value / world / (peak * 1e9 / bytes_per_token), 4),
            "e2e": {"value": round(world * K / te, 2), "unit": UNIT, "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8},
            "greedy_tokens": "identical to the reference CPU backend's (REFERENCE numerics)",
            "gpu_launches": K * (1 + 28 * 5 + 1)}


def run_b200(args):
    import torch
    from wginfer_b200 import numerics
    from wginfer_b200.synthetic import Qwen2Config, prompt_ids

    world, rank, local = dist_setup(args.gpus)
    peak, peak_src = load_peaks()
    K, W = args.steps, args.warmup
    maxseq = args.prompt + W + K + W + K + 8
    cfg = Qwen2Config(nlayer=28, maxseq=maxseq)
    result = {"metric": METRIC, "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
              "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
              "data": "synthetic (seeded random weights ~N(0,0.02), uniform random prompt ids)"}
    with numerics(args.numerics):
        m, kept = build_model(cfg, 1, local, seed=0, keep=("out_embed",))
        m.prefill(0, prompt_ids(args.prompt, cfg.voc, seed=rank).numpy())
        with Clocks(local) as clk:
            t = time_decode(m, 1, K, W, world)
        t_max = max_over_ranks(t, world)
        value = world * K / t_max
        # e2e through the public API: host token in, host token out, every step
        te = time_e2e(m, K, W, world)
        roof = gemv_roofline(kept["out_embed"], cfg, peak)
        roof["peak_source"] = peak_src
        del kept
    bytes_per_token = cfg.weight_bytes()
    ref_leg = None
    if args.numerics == "fast" and not args.no_reference_numerics:
        ref_leg = reference_numerics_leg(m, args, world, rank, bytes_per_token, peak)
    m.close()
    torch.cuda.empty_cache()
    result.update({
        "value": round(value, 2), "ms_per_step": round(t_max / K * 1e3, 4),
        "config": decode_config(args, world),
        "weight_stream_roofline": {"bytes_per_token": bytes_per_token,
                                   "tok_s_at_peak": round(peak * 1e9 / bytes_per_token, 1),
                                   "frac": round(value / world / (peak * 1e9 / bytes_per_token), 4)},
        "e2e": {"value": round(world * K / te, 2), "unit": UNIT, "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8},
        "roofline": roof,
        "clocks": clk.summary(),
        # per step: embedding, 28 x (qkv gemv [rms, rope, kv append fused], attention,
        # o gemv [+residual], gate/up gemv [rms, swiglu fused], down gemv [+residual]), lm_head gemv
        # [final rms, greedy argmax and sequence lengths advanced, fused]
        "gpu_launches": K * (1 + 28 * 5 + 1),
    })
    # the long sweep first; the batched and REFERENCE results close the line
    # (a reader of its last characters sees them)
    if rank == 0 and not args.no_sweep:
        result["op_bandwidth"] = op_sweep(peak, quick=world > 1)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(args.cpu_steps)
    if rank == 0 and world == 1 and not args.no_prefill:
        try:
            result["prefill"] = prefill_only(args.prompt, 3)
        except Exception as e:  # a side measurement: the decode line is still printed
            result["prefill"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if not args.no_bs64:
        result["bs64"] = bs64(args, world, rank, local)
    if ref_leg is not None:
        result["reference_numerics"] = ref_leg
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def bs64(args, world, rank, local):
    """64 sequences x 2048-token prompts, 256-token decode budget, on the
    one-layer model; each GPU holds 64/N of them."""
    from wginfer_b200 import numerics
    from wginfer_b200.synthetic import Qwen2Config, prompt_ids
    from wginfer_b200 import dist as D
    total = 64
    mine = D.partition(total, world, rank)  # this GPU's requests
    per = len(mine)
    K, W = min(args.steps, 200), min(args.warmup, 8)
    cfg = Qwen2Config(nlayer=1, maxseq=2048 + 256)
    with numerics(args.numerics):
        m, _ = build_model(cfg, per, local, seed=0)
        ids = prompt_ids(2048, cfg.voc, seed=1000, batch=total).numpy()
        t0 = time.time()
        for b, i in enumerate(mine):
            m.prefill(b, ids[i])
        prefill_s = time.time() - t0
        t = time_decode(m, per, K, W, world)
        m.close()
    t_max = max_over_ranks(t, world)
    # HBM bytes one GPU's step must move: every weight once (the layer, the
    # final norm, lm_head) and its sequences' K/V (2 x 2 heads x 128 x 2 B
    # per cached position) at the mean cache length of the timed steps
    peak, _ = load_peaks()
    cache = 2048 + W + K / 2
    step_bytes = cfg.weight_bytes() + per * cache * 2 * cfg.nkvh * cfg.dh * 2
    return {"value": round(total * K / t_max, 1), "unit": UNIT, "sequences": total, "per_gpu": per,
            "prompt": 2048, "steps": K, "ms_per_step": round(t_max / K * 1e3, 4), "scaling": "strong",
            "hbm_frac": round(step_bytes / (t_max / K) / 1e9 / peak, 3), "prefill_s_rank0": round(prefill_s, 2),
            "workload": "one-layer Qwen2 (the config-2 layer + embeddings + lm_head), bf16, greedy"}


def prefill_only(plen: int, reps: int) -> dict:
    """One sequence's prefill of `plen` tokens on the 28-layer model (FAST
    numerics, one GPU): CUDA events on the model's stream around
    wgb_qwen2_prefill, the best of `reps` after one warm-up."""
    import torch
    from wginfer_b200 import numerics
    from wginfer_b200.synthetic import Qwen2Config, prompt_ids
    cfg = Qwen2Config(nlayer=28, maxseq=plen + 64)
    with numerics("fast"):
        m, _ = build_model(cfg, 1, 0)
        ids = prompt_ids(plen, cfg.voc, seed=0).numpy()
        st = m.torch_stream()
        times = []
        for r in range(reps + 1):
            m.reset_cache()
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(st)
            m.prefill(0, ids)
            e.record(st)
            torch.cuda.synchronize()
            if r:
                times.append(s.elapsed_time(e) / 1e3)
        m.close()
    best = min(times)
    return {"prompt": plen, "value": round(plen / best, 1), "unit": "tok/s", "ms": round(best * 1e3, 3),
            "reps": reps, "workload": "28-layer Qwen2-1.5B architecture, bf16, FAST, one sequence"}


# ---------------------------------------------------------------- reference CPU arm
def reference_model():
    """The reference's own Model (oracle/_ref, its CPU device) with the
    28-layer Qwen2-1.5B architecture and the same seeded weights the tests
    use (~3 GB of bf16 on the host)."""
    from oracle import oracle as O
    from tests.golden import cases as CS
    from wginfer_b200.synthetic import Qwen2Config
    cfg = Qwen2Config(nlayer=28, maxseq=256)
    meta, w = CS.model_inputs(cfg, seed=0)
    m = O.ReferenceQwen2(O.Reference(), meta, w)
    del w
    return m


def reference_decode_times(steps: int, warmup: int):
    """Seconds per decode token of the reference Model::infer, batch 1, for
    `steps` tokens after `warmup` untimed ones. The prompt is one token, so
    the cache holds 1..steps+warmup+1 positions (a longer prompt would need a
    prefill that forms logits for every prompt row, minutes on the CPU;
    attention over 512 positions is under 1% of the CPU token time, which is
    the linears')."""
    import numpy as np
    m = reference_model()
    tok = m.infer(np.array([1], np.int64))
    for _ in range(warmup):
        tok = m.infer(np.array([tok], np.int64))
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        tok = m.infer(np.array([tok], np.int64))
        times.append(time.perf_counter() - t0)
    del m
    return times


REF_SAMPLE = ("decode tokens of the reference Model::infer (oracle/_ref, the full 28-layer Qwen2-1.5B "
              "architecture on its CPU device, batch 1, greedy), prompt 1 token, cache 1..%d positions; "
              "its linear is single-threaded below 64 rows")


def cpu_baseline(steps: int):
    try:
        from oracle import oracle as O
        if not os.path.exists(O.REF_SO):
            return {"value": None, "unavailable": "oracle/_ref not built"}
        per = reference_decode_times(steps, warmup=1)
        v = len(per) / sum(per)
        return {"value": round(v, 4), "unit": UNIT, "cores": os.cpu_count(), "kind": "reference",
                "sample": f"{len(per)} " + REF_SAMPLE % (len(per) + 2)}
    except Exception as e:  # reported, never fatal for the GPU arm
        return {"value": None, "unavailable": f"{type(e).__name__}: {e}"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from oracle import oracle as O
    if not os.path.exists(O.REF_SO):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref (reference CPU build) missing"}))
        return
    K, W = args.steps, args.warmup
    per = reference_decode_times(K, W)
    t = sum(per)
    value = K / t
    cores = os.cpu_count()
    config = {"workload": "Qwen2-1.5B arch (28 layers, hidden 1536, 12/2 heads x 128, MLP 8960, vocab 151936), "
                          "greedy decode, batch 1, reference CPU Model, prompt 1 token",
              "global_batch": 1, "seq_len": 1 + W + K + 1, "parallelism": "one host process (rank 0)",
              "numerics": "the reference's own", "l2": "n/a (CPU)"}
    out = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world,
           "steps": K, "warmup": W, "ms_per_step": round(t / K * 1e3, 2),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic (seeded random weights)", "config": config,
           "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": cores, "kind": "reference",
                            "sample": f"{K} " + REF_SAMPLE % (W + K + 1)},
           "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--numerics", default="fast", choices=["fast", "reference"])
    ap.add_argument("--no-bs64", action="store_true")
    ap.add_argument("--only-bs64", action="store_true",
                    help="print only the batched-decode result (64 sequences x 2048-token prompts)")
    ap.add_argument("--only-prefill", type=int, default=0, metavar="TOKENS",
                    help="print only the time of one prefill of this many tokens (28-layer model, one GPU)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the one-GPU prefill timing of the --prompt tokens (28-layer model)")
    ap.add_argument("--op-probe", choices=["add", "swiglu", "rms_norm", "argmax"], default=None,
                    help="only launch one swept op a few times at >= 64 MB (for an ncu capture)")
    ap.add_argument("--no-reference-numerics", action="store_true",
                    help="skip the REFERENCE-numerics (token-identical) decode measurement")
    ap.add_argument("--no-sweep", action="store_true", help="skip the elementwise/reduction bandwidth sweep")
    ap.add_argument("--cpu-steps", type=int, default=2,
                    help="decode tokens of the reference CPU Model timed for cpu_baseline (~6 s each)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.op_probe:
        op_probe(args.op_probe)
    elif args.only_prefill:
        print(json.dumps({"metric": "prefill tok/s", "prefill": prefill_only(args.only_prefill, max(1, args.steps))}),
              flush=True)
    elif args.impl == "reference":
        run_reference(args)
    elif args.only_bs64:
        world, rank, local = dist_setup(args.gpus)
        r = bs64(args, world, rank, local)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"metric": METRIC, "unit": UNIT, "n_gpus": world, "bs64": r}), flush=True)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
