"""The multi-GPU build of the library (ungx_cross_edges_build_distributed), through the C ABI.

* A world of one (no communicator, and a one-rank NCCL communicator) reproduces the
  golden fixtures from host slices and from device-resident vectors, and the second
  call with the same problem reuses the plan.
* With two or more GPUs: one process per GPU, NCCL ids handed over by the parent; the
  slices uploaded per rank, replicated over NVLink, the shards gathered on rank 0 --
  rank 0's output equals the single-GPU result and the fixtures.  Skipped on boxes
  with one GPU.
"""
import multiprocessing as mp
import os

import numpy as np
import pytest

from conftest import load_golden
from filtervectorcode_refactor_b200 import _native as nat
from parity import assert_rows_match

pytestmark = pytest.mark.gpu


def golden_problem(g, route=nat.ROUTE_AUTO):
    n, d = g["Xr"].shape
    return nat.Problem(n, d, g["k"], g["group_ranges"], g["out_offsets"], g["out_ids"], route=route)


def test_world_of_one_host_slices(golden):
    n, d = golden["Xr"].shape
    k = golden["k"]
    prob = golden_problem(golden)
    with nat.Context(0) as ctx:
        for call in range(2):
            ids = np.full(n * k, 5, dtype=np.uint32)
            dists = np.full(n * k, -1, dtype=np.float32)
            t = ctx.build_distributed(golden["Xr"], prob, ids, dists)
            assert_rows_match(ids, dists, golden["ids"], golden["dists"], k)
            assert t.world_size == 1 and t.shard_rows == n
            assert t.plan_reused == (1 if call else 0)


def test_world_of_one_device_vectors_and_output(golden):
    import torch
    n, d = golden["Xr"].shape
    k = golden["k"]
    prob = golden_problem(golden)
    X = torch.from_numpy(golden["Xr"]).cuda()
    d_ids = torch.empty(n * k, dtype=torch.int32, device="cuda")
    d_dists = torch.empty(n * k, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    with nat.Context(0) as ctx:
        ctx.build_distributed(X.data_ptr(), prob, d_ids.data_ptr(), d_dists.data_ptr(),
                              nat.DIST_DEVICE_VECTORS | nat.DIST_DEVICE_OUTPUT)
    assert_rows_match(d_ids.cpu().numpy().view(np.uint32), d_dists.cpu().numpy(), golden["ids"], golden["dists"], k)


def test_one_rank_communicator():
    g = load_golden("cfg2_n6000")
    n, d = g["Xr"].shape
    k = g["k"]
    ids = np.empty(n * k, dtype=np.uint32)
    dists = np.empty(n * k, dtype=np.float32)
    with nat.Context(0) as ctx:
        ctx.comm_init(nat.comm_id_create(), 1, 0)
        t = ctx.build_distributed(g["Xr"], golden_problem(g), ids, dists)
        ctx.comm_destroy()
    assert t.world_size == 1
    assert_rows_match(ids, dists, g["ids"], g["dists"], k)


def _rank_main(rank, world, comm_id, case, device_vectors, out_q):
    """One rank of a multi-GPU build (a spawned process with its own GPU)."""
    try:
        import numpy as np  # noqa: F811
        import torch  # its NCCL first: the library then uses the copy already loaded
        from filtervectorcode_refactor_b200 import _native as nat  # noqa: F811
        Xr, k, ranges, off, ids_lng = case
        n, d = Xr.shape
        prob = nat.Problem(n, d, k, ranges, off, ids_lng)
        ctx = nat.Context(rank)
        ctx.set_timeout_ms(120000)
        ctx.comm_init(comm_id, world, rank)
        out_ids = np.empty(n * k, dtype=np.uint32) if rank == 0 else None
        out_d = np.empty(n * k, dtype=np.float32) if rank == 0 else None
        timings = []
        for _ in range(2):
            if device_vectors:
                torch.cuda.set_device(rank)
                X = torch.from_numpy(Xr).cuda()
                torch.cuda.synchronize()
                t = ctx.build_distributed(X.data_ptr(), prob, out_ids, out_d, nat.DIST_DEVICE_VECTORS)
            else:
                a, c = nat.dist_slice(n, world, rank)
                t = ctx.build_distributed(np.ascontiguousarray(Xr[a:a + c]), prob, out_ids, out_d)
            timings.append(t.as_dict())
        ctx.comm_destroy()
        ctx.close()
        out_q.put((rank, "ok", out_ids, out_d, timings))
    except Exception as e:  # reported to the parent, which fails the test
        out_q.put((rank, f"error: {e!r}", None, None, None))


def run_ranks(world, case, device_vectors=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    comm_id = nat.comm_id_create()
    procs = [ctx.Process(target=_rank_main, args=(r, world, comm_id, case, device_vectors, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r, status, ids, dists, timings = q.get(timeout=300)
            results[r] = (status, ids, dists, timings)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert results[r][0] == "ok", f"rank {r}: {results[r][0]}"
    return results


def gpu_count():
    import torch
    return torch.cuda.device_count()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("device_vectors", [False, True], ids=["host_slices", "device_vectors"])
def test_multi_gpu_build_matches_golden(world, device_vectors):
    if gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    for name in ("cfg2_n6000", "cfg4_n6000", "edge_ties_k40"):
        g = load_golden(name)
        case = (g["Xr"], g["k"], g["group_ranges"], g["out_offsets"], g["out_ids"])
        res = run_ranks(world, case, device_vectors)
        status, ids, dists, timings = res[0]
        assert_rows_match(ids, dists, g["ids"], g["dists"], g["k"])
        n = g["Xr"].shape[0]
        assert sum(res[r][3][-1]["shard_rows"] for r in range(world)) == n
        assert all(res[r][3][-1]["plan_reused"] == 1 for r in range(world))


def test_multi_gpu_build_config2_scale():
    """200,000 points of configuration 2 on two GPUs: rank 0's gathered output equals the
    single-GPU build of the same problem on every row."""
    if gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    from filtervectorcode_refactor_b200 import datasets
    c = datasets.make_config(2, seed=5, n=200_000)
    lg = nat.LabelGraph(c["label_offsets"], c["labels"])
    Xr = datasets.reorder_rows(c["X"], lg.new_to_old)
    n, d, k = Xr.shape[0], Xr.shape[1], c["k"]
    ref_ids = np.empty(n * k, dtype=np.uint32)
    ref_d = np.empty(n * k, dtype=np.float32)
    with nat.Context(0) as ctx:
        ctx.build(Xr, nat.Problem(n, d, k, lg.group_ranges, lg.out_offsets, lg.out_ids), ref_ids, ref_d)
    res = run_ranks(2, (Xr, k, lg.group_ranges, lg.out_offsets, lg.out_ids))
    assert_rows_match(res[0][1], res[0][2], ref_ids, ref_d, k)
