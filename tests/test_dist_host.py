"""CPU, multi-process (gloo): the head sharding and verification gather used for 1..8 GPUs, plus host-side
failure detection (a rank that never joins makes the others fail fast instead of hanging).

Each rank generates only its own heads (seeded per global head), computes them with the oracle as the
stand-in for the GPU kernel, and rank 0 gathers; the result must equal the single-process run exactly.
"""
import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cuda_attn.workloads import Config, head_range, make_inputs

SMALL = Config("small", 2, 3, 40, 16, torch.float32, std=0.7, k_outlier_frac=0.05)


@pytest.mark.parametrize("total", [1, 5, 32, 128])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_head_range_partitions_exactly(total, world):
    seen = []
    for r in range(world):
        a, b = head_range(total, world, r)
        assert 0 <= a <= b <= total
        seen += list(range(a, b))
    assert seen == list(range(total))
    sizes = [b - a for a, b in (head_range(total, world, r) for r in range(world))]
    assert max(sizes) - min(sizes) <= 1


def test_head_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        head_range(8, 2, 2)


def test_per_head_seeding_reproduces_single_process_inputs():
    full = make_inputs(SMALL, device="cpu")
    for world in (2, 4):
        for r in range(world):
            a, b = head_range(SMALL.BH, world, r)
            part = make_inputs(SMALL, heads=(a, b), device="cpu")
            for x, y in zip(full, part):
                assert torch.equal(x.reshape(SMALL.BH, SMALL.N, SMALL.d)[a:b], y[0])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, result_q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        from cuda_attn.dist import gather_heads
        from oracle import attention_naive
        a, b = head_range(SMALL.BH, world, rank)
        q, k, v = make_inputs(SMALL, heads=(a, b), device="cpu")
        o = torch.from_numpy(attention_naive(q.numpy(), k.numpy(), v.numpy()).astype(np.float32))
        if mode == "rank1_dies" and rank == 1:
            result_q.put((rank, "exited"))
            result_q.close()
            result_q.join_thread()
            os._exit(0)  # leaves between steps, no collective in flight
        full = gather_heads(o, SMALL.BH, world, rank)
        if rank == 0:
            q, k, v = make_inputs(SMALL, device="cpu")
            ref = attention_naive(q.numpy(), k.numpy(), v.numpy()).astype(np.float32)
            ok = torch.equal(full[0], torch.from_numpy(ref).reshape(SMALL.BH, SMALL.N, SMALL.d))
            result_q.put((rank, "equal" if ok else "mismatch"))
        else:
            result_q.put((rank, "sent"))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent; a collective error is an expected outcome
        result_q.put((rank, f"error: {type(e).__name__}: {str(e).splitlines()[0][:200]}"))
        traceback.print_exc()


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    out = {}
    while not q.empty():
        r, msg = q.get()
        out[r] = msg
    return out


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_run_gathers_to_single_process_result(world):
    out = _run(world, "normal")
    assert out.get(0) == "equal", out
    assert all(out.get(r) == "sent" for r in range(1, world)), out


def test_rank_that_never_joins_fails_fast():
    out = _run(2, "rank1_dies")
    assert out.get(1) == "exited"
    assert out.get(0, "").startswith("error"), out
