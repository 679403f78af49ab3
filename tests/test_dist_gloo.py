"""Host logic of the batch-sharded multi-GPU path, run as gloo ranks on CPU.

The CUDA operators are not called here; each rank runs the CPU oracle on its
batch slice (the same sharding the GPU ranks use), the slices are assembled
with gather_batch, and the result must equal the unsharded computation.
Failure detection: a rank that raises before a collective makes the others
fail within the process-group timeout instead of hanging.
"""

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from ascendc_kernel_b200 import dist as dd


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, fn, result_q, timeout_s):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    try:
        dd.init(backend="gloo", timeout_s=timeout_s)
        out = fn(rank, world)
        result_q.put((rank, "ok", out))
    except Exception as exc:  # reported to the parent, never swallowed
        result_q.put((rank, "error", f"{type(exc).__name__}: {exc}\n{traceback.format_exc()}"))
    finally:
        if torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


def run_ranks(fn, world=2, timeout_s=30.0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, q, timeout_s))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, payload = q.get(timeout=timeout_s * 4)
        results[rank] = (status, payload)
    for p in procs:
        p.join(timeout=timeout_s * 2)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("n,world", [(8, 2), (7, 2), (3, 4), (1, 2), (0, 3), (16, 8)])
def test_shard_range_partitions(n, world):
    seen = []
    for r in range(world):
        a, b = dd.shard_range(n, r, world)
        assert 0 <= a <= b <= n
        seen.extend(range(a, b))
    assert seen == list(range(n))
    sizes = [b - a for a, b in (dd.shard_range(n, r, world) for r in range(world))]
    assert max(sizes) - min(sizes) <= 1


def _sharded_sparse_attn(rank, world):
    import oracle
    g = torch.Generator().manual_seed(5)
    B, M, H, D = 5, 6, 16, 128
    q = torch.randn(B, M, H, D, generator=g).to(torch.bfloat16)
    kv = torch.randn(B, 32, D, generator=g).to(torch.bfloat16)
    idx = torch.randint(0, 32, (B, M, 16), generator=g, dtype=torch.int32)
    u16 = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)
    qs, kvs, ids = (dd.shard_batch(t, rank, world) for t in (q, kv, idx))
    out = oracle.sparse_attn(u16(qs), u16(kvs), ids.numpy(), np.zeros(H, np.float32), D ** -0.5)
    shard = torch.from_numpy(out.view(np.int16))
    full = dd.gather_batch(shard, B)
    want = oracle.sparse_attn(u16(q), u16(kv), idx.numpy(), np.zeros(H, np.float32), D ** -0.5)
    slowest = dd.max_over_ranks(float(rank + 1))
    return bool(np.array_equal(full.numpy().view(np.uint16), want)), slowest


def test_sharded_forward_equals_unsharded_gloo():
    res = run_ranks(_sharded_sparse_attn, world=2)
    for rank, (status, payload) in res.items():
        assert status == "ok", payload
        equal, slowest = payload
        assert equal
        assert slowest == 2.0


def _one_rank_fails(rank, world):
    if rank == 1:
        raise RuntimeError("injected failure on rank 1 before the gather")
    dd.gather_batch(torch.zeros(2, 3), 4)
    return "unreachable"


def test_failed_rank_is_detected_not_hung():
    res = run_ranks(_one_rank_fails, world=2, timeout_s=10.0)
    assert res[1][0] == "error" and "injected failure" in res[1][1]
    # rank 0 must end with an error (peer gone / timeout), not hang or succeed
    assert res[0][0] == "error", res[0]
