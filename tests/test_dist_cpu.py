"""Rank logic of batched decode partitioned by request (wginfer_b200/dist.py),
on CPU with the gloo backend and world_size 2: request slices, the max over
ranks of a timed region, gathering token streams to rank 0, and a rank that
fails making its peer fail within the process-group timeout instead of
hanging. The GPU replicas themselves are exercised by bench.py --gpus N."""
import os
import socket
import traceback

import numpy as np
import pytest
import torch.multiprocessing as mp

from wginfer_b200 import dist as D


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _fake_stream(prompt, steps):
    # a deterministic "decoder": token t of a request is a hash of its prompt and t
    base = int(np.asarray(prompt, np.int64).sum()) % 1000
    return np.array([(base * 31 + t * 7) % 151936 for t in range(steps)], np.int64)


def _run_slice(prompts, steps):
    return np.stack([_fake_stream(p, steps) for p in prompts]) if prompts else np.empty((0, steps), np.int64)


def _worker(rank, world, port, case, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    try:
        timeout = 3.0 if case == "failure" else 60.0
        w, r, _ = D.setup(backend="gloo", timeout_s=timeout)
        assert (w, r) == (world, rank)
        if case == "collectives":
            t = D.max_over_ranks(1.5 + rank)
            prompts = [np.arange(i + 1) for i in range(5)]
            got = D.decode_requests(prompts, 4, _run_slice)
            D.barrier()
            q.put((rank, "ok", t, None if got is None else got.tolist()))
        elif case == "failure":
            if rank == 1:
                raise RuntimeError("rank 1 fails before the gather")
            try:
                D.gather_streams(np.zeros((1, 2), np.int64), 2)
                q.put((rank, "no error", None, None))
            except Exception as e:  # the peer never joins: the collective must fail, not hang
                q.put((rank, "peer failure seen", type(e).__name__, None))
    except Exception as e:
        q.put((rank, "error", f"{type(e).__name__}: {e}", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(case, world=2, wait=90):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = {}
    for _ in range(world):
        rank, status, a, b = q.get(timeout=wait)
        out[rank] = (status, a, b)
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("n,world", [(64, 1), (64, 2), (64, 8), (5, 2), (3, 4), (0, 2), (7, 3)])
def test_partition_covers_every_request_once(n, world):
    slices = [D.partition(n, world, r) for r in range(world)]
    assert [i for s in slices for i in s] == list(range(n))
    sizes = [len(s) for s in slices]
    assert max(sizes) - min(sizes) <= 1


def test_partition_rejects_bad_arguments():
    with pytest.raises(ValueError):
        D.partition(4, 0, 0)
    with pytest.raises(ValueError):
        D.partition(4, 2, 2)


def test_single_process_decode_requests():
    prompts = [np.arange(i + 1) for i in range(5)]
    got = D.decode_requests(prompts, 4, _run_slice)
    assert np.array_equal(got, _run_slice(prompts, 4))


def test_two_ranks_gather_and_max():
    out = _run("collectives")
    assert out[0][0] == "ok" and out[1][0] == "ok", out
    assert out[0][1] == out[1][1] == 2.5  # max over ranks of 1.5 + rank
    prompts = [np.arange(i + 1) for i in range(5)]
    assert np.array_equal(np.array(out[0][2]), _run_slice(prompts, 4))  # rank 0 holds every stream, in order
    assert out[1][2] is None


def test_failed_rank_makes_peer_fail_not_hang():
    out = _run("failure", wait=120)
    assert out[1][0] == "error" and "rank 1 fails" in out[1][1]
    assert out[0][0] == "peer failure seen", out[0]
