"""Additional edges and device-side graph emission, through the C ABI.

* ungx_additional_edges_build on the device cross-edge output reproduces the
  reference's additional edges (exact variant of build_cross_edges_generate_additional,
  golden fixtures made by the reference's compiled code): the (from, to) list in the
  reference's order, and the same edges per point;
* ungx_graph_csr_device emits, per point, intra-group edges, then cross edges in queue
  order, then additional edges, equal to the same adjacency assembled on the host;
* a column buffer that is too small is refused without writing;
* ungx_build_cross_group_edges (generate, additional edges, add_offset and merge in one
  call) equals the reference's per-point adjacency assembled from the fixtures.
"""
import numpy as np
import pytest

from filtervectorcode_refactor_b200 import _native as nat
from graph_case import expected_merged_graph, local_intra_graph

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ctx():
    c = nat.Context(0)
    yield c
    c.close()


def cross_on_device(ctx, g):
    n, d = g["Xr"].shape
    k = g["k"]
    route = nat.ROUTE_TENSOR if k <= 24 else nat.ROUTE_EXACT
    prob = nat.Problem(n, d, k, g["group_ranges"], g["out_offsets"], g["out_ids"], route=route)
    ctx.prepare_base_vectors(g["Xr"], n, d, on_device=False)
    d_ids = torch.empty((n, k), dtype=torch.int32, device="cuda")
    d_dists = torch.empty((n, k), dtype=torch.float32, device="cuda")
    ctx.generate_device(prob, d_ids.data_ptr(), d_dists.data_ptr())
    torch.cuda.synchronize()
    return prob, d_ids


def test_additional_edges_match_golden(ctx, golden):
    prob, d_ids = cross_on_device(ctx, golden)
    n = golden["Xr"].shape[0]
    assert np.array_equal(d_ids.cpu().numpy().view(np.uint32).ravel(), golden["ids"])
    st = ctx.additional_edges(prob, d_ids.data_ptr())
    src, dst, off, cols = ctx.additional_edges_copy(n, int(st.edges))
    ctx.release_base_vectors()
    assert np.array_equal(src, golden["add_from"])
    assert np.array_equal(dst, golden["add_to"])
    # per point: the same edges, in list order
    exp_off = np.zeros(n + 1, dtype=np.uint64)
    np.add.at(exp_off, golden["add_from"].astype(np.int64) + 1, 1)
    exp_off = np.cumsum(exp_off).astype(np.uint64)
    assert np.array_equal(off, exp_off)
    order = np.argsort(golden["add_from"], kind="stable")
    assert np.array_equal(cols, golden["add_to"][order])
    assert st.edges == golden["add_from"].size
    assert st.missing_group_edges >= (1 if st.edges else 0)


def test_graph_csr_device_matches_host_assembly(ctx, golden):
    prob, d_ids = cross_on_device(ctx, golden)
    n = golden["Xr"].shape[0]
    k = golden["k"]
    st = ctx.additional_edges(prob, d_ids.data_ptr())
    _, _, add_off, add_cols = ctx.additional_edges_copy(n, int(st.edges))
    ctx.release_base_vectors()
    rng = np.random.default_rng(n)
    deg = rng.integers(0, 6, size=n)
    intra_off = np.zeros(n + 1, dtype=np.uint64)
    intra_off[1:] = np.cumsum(deg)
    intra_cols = rng.integers(0, n, size=int(intra_off[-1])).astype(np.uint32)
    ids = golden["ids"].reshape(n, k)
    expected = []
    for v in range(n):
        row = list(intra_cols[intra_off[v]:intra_off[v + 1]])
        row += [x for x in ids[v] if x != 0xFFFFFFFF]
        row += list(add_cols[add_off[v]:add_off[v + 1]])
        expected.append(row)
    exp_off = np.zeros(n + 1, dtype=np.uint64)
    exp_off[1:] = np.cumsum([len(r) for r in expected])
    exp_cols = np.array([x for r in expected for x in r], dtype=np.uint32)

    d_intra_off = torch.from_numpy(intra_off.view(np.int64)).cuda()
    d_intra_cols = torch.from_numpy(intra_cols.view(np.int32) if intra_cols.size else np.zeros(1, np.int32)).cuda()
    d_off = torch.empty(n + 1, dtype=torch.int64, device="cuda")
    cap = int(exp_off[-1])
    d_cols = torch.empty(max(cap, 1), dtype=torch.int32, device="cuda")
    # too small a column buffer is refused
    if cap:
        with pytest.raises(nat.UngxError):
            ctx.graph_csr_device(n, k, d_intra_off.data_ptr(), d_intra_cols.data_ptr(), d_ids.data_ptr(), True,
                                 d_off.data_ptr(), d_cols.data_ptr(), cap - 1)
    total = ctx.graph_csr_device(n, k, d_intra_off.data_ptr(), d_intra_cols.data_ptr(), d_ids.data_ptr(), True,
                                 d_off.data_ptr(), d_cols.data_ptr(), cap)
    assert total == cap
    assert np.array_equal(d_off.cpu().numpy().view(np.uint64), exp_off)
    assert np.array_equal(d_cols.cpu().numpy().view(np.uint32)[:cap], exp_cols)
    # cross edges alone: the CSR of build_csr_adjacency
    total2 = ctx.graph_csr_device(n, k, None, None, d_ids.data_ptr(), False, d_off.data_ptr(), d_cols.data_ptr(),
                                  cap)
    h_off, h_cols = nat.flat_to_csr(golden["ids"], n, k)
    assert total2 == int(h_off[-1])
    assert np.array_equal(d_off.cpu().numpy().view(np.uint64), h_off)
    assert np.array_equal(d_cols.cpu().numpy().view(np.uint32)[:total2], h_cols)


@pytest.mark.parametrize("additional", [True, False], ids=["with_additional", "cross_only"])
def test_build_cross_group_edges_one_call(ctx, golden, additional):
    """ungx_build_cross_group_edges (the whole build_cross_group_edges step: generate,
    additional edges, add_offset, merge) equals the reference's per-point adjacency
    assembled from the golden fixtures."""
    n, d = golden["Xr"].shape
    k = golden["k"]
    route = nat.ROUTE_TENSOR if k <= 24 else nat.ROUTE_EXACT
    prob = nat.Problem(n, d, k, golden["group_ranges"], golden["out_offsets"], golden["out_ids"], route=route)
    intra_off, intra_cols = local_intra_graph(golden, n)
    flags = nat.BUILD_INTRA_LOCAL_IDS | (nat.BUILD_ADDITIONAL if additional else 0)
    ids = np.empty(n * k, dtype=np.uint32)
    dists = np.empty(n * k, dtype=np.float32)
    st = ctx.build_cross_group_edges(golden["Xr"], prob, intra_off, intra_cols, flags, ids, dists)
    off, cols = ctx.graph_copy(n, int(st.num_cols))
    ctx.release_base_vectors()
    assert np.array_equal(ids, golden["ids"])
    assert np.array_equal(dists.view(np.uint32), golden["dists"].view(np.uint32))
    e_off, e_cols = expected_merged_graph(golden, intra_off, intra_cols, additional)
    assert np.array_equal(off, e_off)
    assert np.array_equal(cols, e_cols)
    assert st.cross_edges == int((golden["ids"] != 0xFFFFFFFF).sum())
    assert st.additional.edges == (golden["add_from"].size if additional else 0)


def test_build_cross_group_edges_device_vectors_global_ids(ctx, golden):
    """Vectors already in device memory and intra columns that are global ids (no offset)."""
    n, d = golden["Xr"].shape
    k = golden["k"]
    if k > 24:
        pytest.skip("tensor route needs k <= 24")
    prob = nat.Problem(n, d, k, golden["group_ranges"], golden["out_offsets"], golden["out_ids"])
    intra_off, intra_local = local_intra_graph(golden, n + 1)
    first = golden["group_first"].astype(np.int64)
    grp = np.searchsorted(first[1:], np.arange(n), side="right")
    intra_global = (intra_local + np.repeat(first[grp], np.diff(intra_off.astype(np.int64)))).astype(np.uint32)
    X = torch.from_numpy(golden["Xr"]).cuda()
    torch.cuda.synchronize()
    st = ctx.build_cross_group_edges(X.data_ptr(), prob, intra_off, intra_global,
                                     nat.BUILD_ADDITIONAL | nat.BUILD_VECTORS_ON_DEVICE)
    off, cols = ctx.graph_copy(n, int(st.num_cols))
    ctx.release_base_vectors()
    e_off, e_cols = expected_merged_graph(golden, intra_off, intra_local, True)
    assert np.array_equal(off, e_off) and np.array_equal(cols, e_cols)


@pytest.mark.parametrize("d", [3, 13, 64, 98, 130, 259])
def test_additional_edges_random_dims(ctx, d):
    """Additional edges of a configuration-2 label structure (6,000 points) over random
    vectors of dimension d, against the C restatement of the reference's exact variant:
    the query kernel's staged row scan at ragged dimensions, copy widths 4 and 16 bytes."""
    import oracle as O
    from filtervectorcode_refactor_b200 import datasets

    c = datasets.make_config(2, seed=7 + d, n=6000)
    lg = nat.LabelGraph(c["label_offsets"], c["labels"])
    gf = np.concatenate([[0], lg.group_ranges[2::2], [lg.group_ranges[-1]]]).astype(np.uint32)
    n, k = 6000, c["k"]
    rng = np.random.default_rng(d)
    Xr = rng.integers(-40, 40, size=(n, d)).astype(np.float32) / 8  # coarse values: ties
    ids_ref, _, _ = O.oracle().cross_exact(Xr, k, gf, lg.out_offsets, lg.out_ids)
    src_ref, dst_ref = O.oracle().additional_edges(Xr, k, gf, lg.out_offsets, lg.out_ids, ids_ref)
    prob = nat.Problem(n, d, k, lg.group_ranges, lg.out_offsets, lg.out_ids, route=nat.ROUTE_EXACT)
    ctx.prepare_base_vectors(Xr, n, d, on_device=False)
    try:
        d_ids = torch.empty((n, k), dtype=torch.int32, device="cuda")
        d_dists = torch.empty((n, k), dtype=torch.float32, device="cuda")
        ctx.generate_device(prob, d_ids.data_ptr(), d_dists.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(d_ids.cpu().numpy().view(np.uint32).ravel(), ids_ref.ravel())
        st = ctx.additional_edges(prob, d_ids.data_ptr())
        src, dst, _, _ = ctx.additional_edges_copy(n, int(st.edges))
    finally:
        ctx.release_base_vectors()
    assert src_ref.size > 0
    assert np.array_equal(src, src_ref)
    assert np.array_equal(dst, dst_ref)
