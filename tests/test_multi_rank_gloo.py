"""Multi-rank host logic on CPU (gloo, world_size 2): every rank derives the same plan,
takes its shard of work items, computes its rows (here with the CPU oracle, standing
in for the device kernels), and the shards are gathered -- as bench.py does with NCCL.
The assembled result must equal the one-rank result, every row covered exactly once.
A rank that fails raises on the host; the other rank's collective then ends with an
error instead of hanging (short process-group timeout)."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, name, fail_rank, q):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import torch
    import torch.distributed as dist

    import oracle as O
    from conftest import load_golden
    from filtervectorcode_refactor_b200 import _native as nat

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        g = load_golden(name)
        n, d = g["Xr"].shape
        k = g["k"]
        prob = nat.Problem(n, d, k, g["group_ranges"], g["out_offsets"], g["out_ids"], shard_rank=rank,
                           shard_count=world)
        rows = prob.shard_rows()
        if rank == fail_rank:
            raise RuntimeError("injected host failure on rank %d" % rank)
        ids, dists = O.oracle().cross_rows(g["Xr"], k, g["group_first"], g["out_offsets"], g["out_ids"], rows)
        # gather (ids, distance bits) of every shard, padded to the largest shard
        cnt = torch.tensor([rows.size], dtype=torch.int64)
        counts = [torch.zeros_like(cnt) for _ in range(world)]
        dist.all_gather(counts, cnt)
        pad = int(max(c.item() for c in counts))
        buf = torch.zeros((pad, 1 + 2 * k), dtype=torch.int64)
        buf[:rows.size, 0] = torch.from_numpy(rows.astype(np.int64))
        buf[:rows.size, 1:1 + k] = torch.from_numpy(ids.astype(np.int64))
        buf[:rows.size, 1 + k:] = torch.from_numpy(dists.view(np.uint32).astype(np.int64))
        parts = [torch.zeros_like(buf) for _ in range(world)]
        dist.all_gather(parts, buf)
        if rank == 0:
            full_ids = np.full((n, k), 0xFFFFFFFF, dtype=np.uint32)
            full_d = np.full((n, k), np.inf, dtype=np.float32)
            seen = np.zeros(n, dtype=np.int64)
            for r, part in enumerate(parts):
                c = int(counts[r].item())
                p = part[:c].numpy()
                rr = p[:, 0]
                seen[rr] += 1
                full_ids[rr] = p[:, 1:1 + k].astype(np.uint32)
                full_d[rr] = p[:, 1 + k:].astype(np.uint32).view(np.float32)
            q.put(("ok", bool(np.all(seen == 1)), full_ids.ravel(), full_d.ravel()))
        else:
            q.put(("done", rank))
    except Exception as e:  # reported to the parent; the peer's collective errors out
        q.put(("error", rank, repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(name, fail_rank=-1, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, name, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    # every rank posts exactly one message; drain the queue before joining (a child
    # cannot exit while its message is still in the pipe)
    import queue as _queue
    import time
    out, deadline = [], time.time() + 120
    while len(out) < world and time.time() < deadline:
        try:
            out.append(q.get(timeout=1.0))
        except _queue.Empty:
            if not any(p.is_alive() for p in procs):
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("name", ["cfg2_n6000", "edge_ties_k8"])
def test_two_rank_shards_reassemble_the_one_rank_result(name):
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from conftest import load_golden
    from parity import assert_rows_match
    res = _run(name)
    oks = [r for r in res if r[0] == "ok"]
    assert len(oks) == 1, res
    _, covered_once, ids, dists = oks[0]
    assert covered_once
    g = load_golden(name)
    assert_rows_match(ids, dists, g["ids"], g["dists"], g["k"])


def test_rank_failure_is_reported_not_hung():
    res = _run("cfg2_n6000", fail_rank=1)
    errors = [r for r in res if r[0] == "error"]
    assert any(r[1] == 1 and "injected" in r[2] for r in errors), res
