"""ungx_cross_edges_exact_noalloc: the exact route for callers that cannot allocate
device memory (code whose device memory belongs to another allocator, services
whose device footprint must not grow while they serve).

Through the C ABI, two calls in a row of the no-allocation entry point must give
the same rows as the existing entry point (ungx_cross_edges_generate, exact route),
ids equal and distance bits equal, the same tolerance as every other parity test
here.  The device's free memory must not change across those calls (the first call
on the device, which may load the library's module, comes before the measurement),
and one of them runs on a non-default stream.  This file is collected last so that
a failure here cannot hide others.
"""
import numpy as np
import pytest

from conftest import load_golden
from filtervectorcode_refactor_b200 import _native as nat
from parity import assert_rows_match

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["cfg2_n6000", "cfg4_n6000", "edge_ties_k40"])
def test_noalloc_matches_existing_entry_point(name):
    import torch

    g = load_golden(name)
    n, d = g["Xr"].shape
    k = g["k"]
    prob = nat.Problem(n, d, k, g["group_ranges"], g["out_offsets"], g["out_ids"], route=nat.ROUTE_EXACT)
    # existing entry point, host buffers
    ref_ids = np.empty(n * k, dtype=np.uint32)
    ref_d = np.empty(n * k, dtype=np.float32)
    with nat.Context(0) as ctx:
        ctx.build(g["Xr"], prob, ref_ids, ref_d)
    # the caller owns every device buffer; the entry point allocates none
    torch.cuda.set_device(0)
    X = torch.from_numpy(g["Xr"]).cuda()
    ids = torch.empty((n * k,), dtype=torch.int32, device="cuda")
    dists = torch.empty((n * k,), dtype=torch.float32, device="cuda")
    side = torch.cuda.Stream()
    # a first call on this device (it may load the library's module with its array)
    nat.cross_edges_exact_noalloc(prob, X.data_ptr(), ids.data_ptr(), dists.data_ptr())
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info(0)[0]
    results = []
    for call, stream in enumerate([None, side]):
        ids.fill_(-7)
        dists.fill_(-3.0)
        torch.cuda.synchronize()
        nat.cross_edges_exact_noalloc(prob, X.data_ptr(), ids.data_ptr(), dists.data_ptr(),
                                      None if stream is None else stream.cuda_stream)
        torch.cuda.synchronize()
        results.append((ids.cpu().numpy().view(np.uint32).copy(), dists.cpu().numpy().copy()))
    free_after = torch.cuda.mem_get_info(0)[0]
    assert free_after == free_before, f"device free memory changed by {free_before - free_after} bytes"
    for got_ids, got_d in results:
        assert_rows_match(got_ids, got_d, ref_ids, ref_d, k)
    assert_rows_match(results[-1][0], results[-1][1], g["ids"], g["dists"], k)


def test_noalloc_rejects_plans_beyond_its_scratch():
    # 20M source rows with one target: the row list alone needs 160 MB > 64 MiB
    n = 20_000_001
    ranges = np.array([0, 0, 0, n - 1, n - 1, n], dtype=np.uint32)
    off = np.array([0, 0, 1, 1], dtype=np.uint64)
    ids = np.array([2], dtype=np.uint32)
    prob = nat.Problem(n, 4, 3, ranges, off, ids, route=nat.ROUTE_EXACT)
    with pytest.raises(nat.UngxError) as e:
        nat.cross_edges_exact_noalloc(prob, 1 << 40, 1 << 40, None)  # never dereferenced
    assert e.value.status == nat.UNGX_ERR_INVALID_ARG
    assert "at most" in str(e.value)
