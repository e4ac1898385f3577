"""The capacity path of ungx_cross_edges_build (the reference's X-side streaming role,
UNG/codes/src/uni_nav_graph_cross_edges.cpp:402-418): with a device memory limit below
the resident footprint, the call runs passes over pairs of row slices and merges each
pass's exact top-k; the rows must equal the fixtures (made by the reference's compiled
code) and the resident result, ids and distance bits, on both routes."""
import numpy as np
import pytest

from conftest import load_golden
from filtervectorcode_refactor_b200 import _native as nat
from parity import assert_rows_match

pytestmark = pytest.mark.gpu

FIXED = 64 << 20


def budget_for_slices(n, d, k, slices):
    """A device limit below the resident footprint that makes the call cut n rows into
    about `slices` slices (at least three)."""
    resident = nat.resident_bytes(n, d, k)
    per = (resident - FIXED) // n
    m = (n + slices - 1) // slices
    return min(FIXED + n * k * 8 + 2 * per * m + per, resident - 1)  # two slices of m rows fit


@pytest.mark.parametrize("slices", [3, 5, 8])
@pytest.mark.parametrize("route", [nat.ROUTE_AUTO, nat.ROUTE_EXACT], ids=["auto", "exact"])
def test_capacity_passes_match_golden(golden, slices, route):
    n, d = golden["Xr"].shape
    k = golden["k"]
    prob = nat.Problem(n, d, k, golden["group_ranges"], golden["out_offsets"], golden["out_ids"], route=route)
    ids = np.full(n * k, 3, dtype=np.uint32)
    dists = np.full(n * k, -1, dtype=np.float32)
    with nat.Context(0) as ctx:
        ctx.set_device_memory_limit(budget_for_slices(n, d, k, slices))
        t = ctx.build(golden["Xr"], prob, ids, dists)
    assert t.passes >= 3
    assert t.pairs == int(golden["pairs"])
    assert_rows_match(ids, dists, golden["ids"], golden["dists"], k)


def test_capacity_passes_match_resident_config2_scale():
    from filtervectorcode_refactor_b200 import datasets
    c = datasets.make_config(2, seed=9, n=200_000)
    lg = nat.LabelGraph(c["label_offsets"], c["labels"])
    Xr = datasets.reorder_rows(c["X"], lg.new_to_old)
    n, d, k = Xr.shape[0], Xr.shape[1], c["k"]
    prob = nat.Problem(n, d, k, lg.group_ranges, lg.out_offsets, lg.out_ids)
    res_ids = np.empty(n * k, dtype=np.uint32)
    res_d = np.empty(n * k, dtype=np.float32)
    ids = np.empty(n * k, dtype=np.uint32)
    dists = np.empty(n * k, dtype=np.float32)
    with nat.Context(0) as ctx:
        t1 = ctx.build(Xr, prob, res_ids, res_d)
        ctx.set_device_memory_limit(budget_for_slices(n, d, k, 4))
        t2 = ctx.build(Xr, prob, ids, dists)
    assert t1.passes == 1 and t2.passes >= 4
    assert t2.pairs == t1.pairs
    assert_rows_match(ids, dists, res_ids, res_d, k)


def test_capacity_budget_too_small_is_refused():
    g = load_golden("cfg2_n6000")
    n, d = g["Xr"].shape
    prob = nat.Problem(n, d, g["k"], g["group_ranges"], g["out_offsets"], g["out_ids"])
    with nat.Context(0) as ctx:
        ctx.set_device_memory_limit(1 << 20)
        with pytest.raises(nat.UngxError) as e:
            ctx.build(g["Xr"], prob, np.empty(n * g["k"], np.uint32), None)
    assert e.value.status == nat.UNGX_ERR_OOM
