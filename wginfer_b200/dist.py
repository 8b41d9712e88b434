"""Batched decode partitioned by request across the GPUs of one node.

One process per GPU (torchrun). Requests are independent: rank r takes a
contiguous, balanced slice of them, runs its own replica of the model over
its slice, and nothing crosses NVLink on the data path; the only collectives
are the host-side bookkeeping below (a barrier around timed regions, a max
over ranks of the elapsed time, and an all-gather of the finished token
streams to rank 0). The reference serves one request at a time on one
device (src/models/qwen2/model.cpp, Model::infer), so this layer has no
counterpart there.

Backends: "nccl" on GPUs; "gloo" works for every helper here on CPU, which is
how the rank logic is tested.
"""
from __future__ import annotations

import os
from datetime import timedelta
from typing import Callable, Sequence

import numpy as np


def partition(n: int, world: int, rank: int) -> range:
    """Contiguous slice of n requests for `rank`: the first n % world ranks
    take one more, so slice sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world or n < 0:
        raise ValueError(f"partition: n={n} world={world} rank={rank}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def env_world() -> tuple[int, int, int]:
    """(world, rank, local_rank) from the torchrun environment (1, 0, 0 alone)."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def setup(backend: str | None = None, timeout_s: float = 300.0) -> tuple[int, int, int]:
    """Initialises the process group when WORLD_SIZE > 1 (NCCL with each rank
    pinned to its local GPU, unless `backend` says otherwise) and returns
    (world, rank, local_rank). The timeout bounds every collective, so a rank
    that fails makes the others fail instead of waiting for good."""
    import torch
    import torch.distributed as dist
    world, rank, local = env_world()
    if world > 1 and not dist.is_initialized():
        backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
        kw = {"timeout": timedelta(seconds=timeout_s)}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, **kw)
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def _device():
    import torch
    import torch.distributed as dist
    if dist.is_initialized() and dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def barrier() -> None:
    import torch.distributed as dist
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def max_over_ranks(x: float) -> float:
    """The largest x over all ranks (the job's time is its slowest rank's)."""
    import torch
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_streams(local: np.ndarray, n_total: int) -> np.ndarray | None:
    """Collects every rank's [slice, steps] int64 token streams into the
    [n_total, steps] array on rank 0 (None elsewhere); slices are the ones
    `partition` assigns, in rank order."""
    import torch
    import torch.distributed as dist
    local = np.ascontiguousarray(local, dtype=np.int64)
    if not dist.is_initialized() or dist.get_world_size() == 1:
        if local.shape[0] != n_total:
            raise ValueError("gather_streams: one rank must hold every request")
        return local
    world, rank = dist.get_world_size(), dist.get_rank()
    if local.shape[0] != len(partition(n_total, world, rank)):
        raise ValueError(f"gather_streams: rank {rank} holds {local.shape[0]} rows, its slice has "
                         f"{len(partition(n_total, world, rank))}")
    steps = local.shape[1] if local.ndim == 2 else 0
    rows = -(-n_total // world)  # pad every slice to the largest one
    buf = torch.full((rows, steps), -1, dtype=torch.int64, device=_device())
    if local.shape[0]:
        buf[:local.shape[0]] = torch.from_numpy(local).to(buf.device)
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf)
    if rank != 0:
        return None
    out = np.empty((n_total, steps), np.int64)
    for r in range(world):
        sl = partition(n_total, world, r)
        out[sl.start:sl.stop] = parts[r][:len(sl)].cpu().numpy()
    return out


def decode_requests(prompts: Sequence[np.ndarray], steps: int,
                    run_slice: Callable[[Sequence[np.ndarray], int], np.ndarray]) -> np.ndarray | None:
    """Greedy-decodes `steps` tokens for every prompt, each rank running
    `run_slice(its prompts, steps) -> [len, steps] tokens` on its own
    replica; returns all streams on rank 0 (None elsewhere)."""
    import torch.distributed as dist
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    sl = partition(len(prompts), world, rank)
    mine = [prompts[i] for i in sl]
    local = run_slice(mine, steps) if mine else np.empty((0, steps), np.int64)
    return gather_streams(np.asarray(local, np.int64).reshape(len(mine), steps), len(prompts))


def qwen2_slice_runner(model) -> Callable[[Sequence[np.ndarray], int], np.ndarray]:
    """`run_slice` for a wginfer_b200.qwen2.Qwen2 replica whose max_batch is
    at least the slice size: prefills each prompt into its own sequence slot,
    then decodes the whole slice as one batch per step."""
    def run(prompts: Sequence[np.ndarray], steps: int) -> np.ndarray:
        model.reset_cache()
        for b, p in enumerate(prompts):
            model.prefill(b, np.asarray(p, np.int64))
        out = np.empty((len(prompts), steps), np.int64)
        out[:, 0] = model.tokens(len(prompts))
        for t in range(1, steps):
            model.decode_step(len(prompts))
            out[:, t] = model.tokens(len(prompts))
        return out
    return run
