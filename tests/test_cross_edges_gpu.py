"""Parity of the B200 cross-edge build against the oracle, through the C ABI.

* golden fixtures (made by the reference's own compiled code): ids and distance bits equal;
* configurations 2, 3 and 4 at their full size: >= 2,000 rows stratified over every
  source-group size, the largest source group and the rows whose targets include the
  largest group are recomputed by the CPU oracle and must match exactly; every row
  satisfies the size-independent properties (sorted, ids from the union of the
  out-groups, min(k, |union|) edges, sentinels last);
* every operand width class of the tensor-core kernel (two issuers, one issuer,
  streamed source rows) matches the oracle on every row;
* the device-pointer entry point equals the host entry point; sharded calls cover
  every row exactly once and reproduce the one-shard result;
* a pipeline wait that runs out returns UNGX_ERR_TIMEOUT and leaves the context usable.
"""
import numpy as np
import pytest

import oracle as O
from parity import assert_rows_match, check_row_properties_fast
from filtervectorcode_refactor_b200 import _native as nat
from filtervectorcode_refactor_b200 import datasets
from filtervectorcode_refactor_b200.ung import UniNavGraph

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = nat.Context(0)
    yield c
    c.close()


def run_golden(ctx, g, route):
    n, d = g["Xr"].shape
    prob = nat.Problem(n, d, g["k"], g["group_ranges"], g["out_offsets"], g["out_ids"], route=route)
    ids = np.full(n * g["k"], 7, dtype=np.uint32)
    dists = np.full(n * g["k"], -1, dtype=np.float32)
    ctx.prepare_base_vectors(g["Xr"], n, d, on_device=False)
    t = ctx.generate(prob, ids, dists)
    ctx.release_base_vectors()
    return ids, dists, t


@pytest.mark.parametrize("route", [nat.ROUTE_TENSOR, nat.ROUTE_EXACT], ids=["tensor", "exact"])
def test_golden_parity(ctx, golden, route):
    if route == nat.ROUTE_TENSOR and golden["k"] > 24:
        with pytest.raises(nat.UngxError):
            run_golden(ctx, golden, route)
        return
    ids, dists, t = run_golden(ctx, golden, route)
    assert t.route_used == route
    assert t.pairs == int(golden["pairs"])
    assert_rows_match(ids, dists, golden["ids"], golden["dists"], golden["k"])


def test_uninavgraph_mirror_end_to_end(golden):
    """The reference-shaped host API: labels + raw vectors in, SearchQueue content out."""
    ung = UniNavGraph(num_cross_edges=golden["k"])
    ung.build(golden["X"], golden["label_offsets"], golden["labels"])
    try:
        assert np.array_equal(ung._new_to_old_vec_ids, golden["new_to_old"])
        assert_rows_match(ung.cross_group_neighbor_flat_ids, ung.cross_group_neighbor_dists, golden["ids"],
                          golden["dists"], golden["k"])
        off, cols = ung.cross_edges_csr()
        assert int(off[-1]) == int((golden["ids"] != 0xFFFFFFFF).sum())
        # build_cross_group_edges also merged the additional edges after each point's cross edges
        assert int(ung.graph_offsets[-1]) == int(off[-1]) + golden["add_from"].size
        assert ung.additional_edge_count == golden["add_from"].size
    finally:
        ung.close()


def test_device_entry_point_matches_host(ctx, golden):
    import torch
    n, d = golden["Xr"].shape
    k = golden["k"]
    if k > 24:
        pytest.skip("tensor route needs k <= 24")
    prob = nat.Problem(n, d, k, golden["group_ranges"], golden["out_offsets"], golden["out_ids"])
    X = torch.from_numpy(golden["Xr"]).cuda()
    d_ids = torch.empty(n * k, dtype=torch.int32, device="cuda")
    d_dists = torch.empty(n * k, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    ctx.prepare_base_vectors(X.data_ptr(), n, d, on_device=True)
    ctx.generate_device(prob, d_ids.data_ptr(), d_dists.data_ptr())
    ctx.release_base_vectors()
    ids = d_ids.cpu().numpy().view(np.uint32)
    dists = d_dists.cpu().numpy()
    assert_rows_match(ids, dists, golden["ids"], golden["dists"], k)



def test_device_entry_point_on_caller_stream(ctx, golden):
    """Generate on the caller's own stream straight after preparation: the preparation
    kernels run on the context's stream and the call must wait for them."""
    import torch
    n, d = golden["Xr"].shape
    k = golden["k"]
    if k > 24:
        pytest.skip("tensor route needs k <= 24")
    prob = nat.Problem(n, d, k, golden["group_ranges"], golden["out_offsets"], golden["out_ids"])
    X = torch.from_numpy(golden["Xr"]).cuda()
    d_ids = torch.empty(n * k, dtype=torch.int32, device="cuda")
    d_dists = torch.empty(n * k, dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    ctx.prepare_base_vectors(X.data_ptr(), n, d, on_device=True)
    ctx.generate_device(prob, d_ids.data_ptr(), d_dists.data_ptr(), s.cuda_stream)
    s.synchronize()
    ctx.release_base_vectors()
    assert_rows_match(d_ids.cpu().numpy().view(np.uint32), d_dists.cpu().numpy(), golden["ids"], golden["dists"], k)

def test_shards_cover_rows_once(ctx, golden):
    n, d = golden["Xr"].shape
    k = golden["k"]
    route = nat.ROUTE_TENSOR if k <= 24 else nat.ROUTE_EXACT
    ids = np.full(n * k, 0xABCDEF, dtype=np.uint32)
    dists = np.full(n * k, -5, dtype=np.float32)
    ctx.prepare_base_vectors(golden["Xr"], n, d, on_device=False)
    seen = np.zeros(n, dtype=np.int64)
    for r in range(3):
        prob = nat.Problem(n, d, k, golden["group_ranges"], golden["out_offsets"], golden["out_ids"], route=route,
                           shard_rank=r, shard_count=3)
        seen[prob.shard_rows()] += 1
        ctx.generate(prob, ids, dists)
    ctx.release_base_vectors()
    assert np.all(seen == 1)
    assert_rows_match(ids, dists, golden["ids"], golden["dists"], k)


@pytest.mark.parametrize("d,dist", [(64, "normal"), (100, "uniform"), (144, "normal"), (200, "uniform"),
                                    (256, "normal"), (300, "normal")])
def test_operand_widths_match_oracle(ctx, d, dist):
    """Every operand layout of the tensor-core kernel against the oracle, all rows: two MMA
    issuers with resident source rows (padded width <= 128), one issuer with resident
    source rows (<= 256), source rows streamed per chunk (> 256)."""
    n, k = 2500, 6
    off, lab = datasets.make_labels(n, vocab=12, umin=1, umax=3, zipf=1.1, seed=d)
    X = datasets.make_vectors(n, d, dist, normalize=False, seed=d)
    lg = nat.LabelGraph(off, lab)
    Xr = np.ascontiguousarray(X[lg.new_to_old])
    prob = nat.Problem(n, d, k, lg.group_ranges, lg.out_offsets, lg.out_ids, route=nat.ROUTE_TENSOR)
    ids = np.empty(n * k, dtype=np.uint32)
    dists = np.empty(n * k, dtype=np.float32)
    ctx.prepare_base_vectors(Xr, n, d, on_device=False)
    t = ctx.generate(prob, ids, dists)
    ctx.release_base_vectors()
    group_first = np.concatenate([[0], lg.group_ranges[2::2], [lg.group_ranges[-1]]]).astype(np.uint32)
    rows = np.arange(n, dtype=np.uint32)
    o_ids, o_d = O.oracle().cross_rows(Xr, k, group_first, lg.out_offsets, lg.out_ids, rows)
    assert_rows_match(ids, dists, o_ids.ravel(), o_d.ravel(), k)
    assert t.rows_fallback <= 0.01 * (t.rows_certified + t.rows_fallback)


def stratified_rows(group_ranges, out_offsets, out_ids, rng, total=2000):
    """Rows for the full-size checks: every source-group size bucket (singletons .. the
    largest group), the largest source group itself, rows whose targets include the
    largest group, groups without targets, then random rows of groups with targets
    up to `total`."""
    gr = group_ranges.reshape(-1, 2).astype(np.int64)
    sizes = gr[:, 1] - gr[:, 0]
    G = gr.shape[0] - 1
    oo = out_offsets.astype(np.int64)
    has_out = np.zeros(G + 1, dtype=bool)
    has_out[:G + 1] = np.diff(oo[:G + 2]) > 0
    has_out[0] = False
    pick = lambda g, m: rng.integers(gr[g, 0], gr[g, 1], size=m)
    rows = []
    for lo in [1, 2, 8, 64, 512, 4096, 32768, 262144]:
        gs = np.nonzero((sizes >= lo) & (sizes < lo * 8) & has_out)[0]
        for g in rng.choice(gs, size=min(40, gs.size), replace=False) if gs.size else []:
            rows.append(pick(g, 3))
    src = np.nonzero(has_out)[0]
    rows.append(pick(src[np.argmax(sizes[src])], 60))                 # the largest source group
    big = int(np.argmax(sizes[1:])) + 1                               # the largest group
    owners = np.repeat(np.arange(G + 1), np.diff(oo[:G + 2]))
    into_big = np.unique(owners[out_ids.astype(np.int64) == big])
    for g in rng.choice(into_big, size=min(60, into_big.size), replace=False) if into_big.size else []:
        rows.append(pick(g, 4))                                       # rows whose targets hold it
    for g in np.nonzero(~has_out & (sizes > 0))[0][:20]:
        rows.append(pick(g, 1))                                       # rows without targets
    rows = np.unique(np.concatenate(rows))
    w = np.where(has_out, sizes, 0).astype(np.float64)
    while rows.size < total:
        need = total - rows.size
        g = rng.choice(G + 1, size=need, p=w / w.sum())
        rows = np.unique(np.concatenate([rows, gr[g, 0] + (rng.random(need) * sizes[g]).astype(np.int64)]))
    return rows.astype(np.uint32)


def full_size_case(cfg):
    c = datasets.make_config(cfg, seed=0)
    lg = nat.LabelGraph(c["label_offsets"], c["labels"])
    Xr = datasets.reorder_rows(c["X"], lg.new_to_old)
    del c["X"]
    return c, lg, Xr


@pytest.mark.parametrize("cfg", [2, 3, 4])
def test_full_size_configuration_parity(ctx, cfg):
    """Configurations 2 (1M x 128), 3 (1M x 960, k = 16) and 4 (10M x 96) at their full
    size through the C ABI: >= 2,000 stratified rows equal to the oracle's exact scan in
    ids and distance bits, >= 100,000 rows (here every row) with the size-independent
    properties, and the certificate clearing nearly every row."""
    c, lg, Xr = full_size_case(cfg)
    N, d, k = Xr.shape[0], Xr.shape[1], c["k"]
    assert N == datasets.CONFIGS[cfg]["n"]
    prob = nat.Problem(N, d, k, lg.group_ranges, lg.out_offsets, lg.out_ids, route=nat.ROUTE_TENSOR)
    ids = np.empty(N * k, dtype=np.uint32)
    dists = np.empty(N * k, dtype=np.float32)
    ctx.prepare_base_vectors(Xr, N, d, on_device=False)
    t = ctx.generate(prob, ids, dists)
    ctx.release_base_vectors()
    print(f"config {cfg}: rows_certified={t.rows_certified} rows_fallback={t.rows_fallback} "
          f"tc_ms={t.tc_kernel_ms:.1f} pairs={t.pairs}")
    rng = np.random.default_rng(100 + cfg)
    rows = stratified_rows(lg.group_ranges, lg.out_offsets, lg.out_ids, rng)
    assert rows.size >= 2000
    group_first = np.concatenate([[0], lg.group_ranges[2::2], [lg.group_ranges[-1]]]).astype(np.uint32)
    o_ids, o_d = O.oracle().cross_rows(Xr, k, group_first, lg.out_offsets, lg.out_ids, rows)
    assert_rows_match(ids.reshape(N, k)[rows], dists.reshape(N, k)[rows], o_ids, o_d, k)
    checked = check_row_properties_fast(ids, dists, k, lg.group_ranges, lg.out_offsets, lg.out_ids,
                                        np.arange(N))
    assert checked >= 100_000
    assert t.rows_certified + t.rows_fallback > 0
    assert t.rows_fallback <= 0.01 * (t.rows_certified + t.rows_fallback)


def test_wait_timeout_reports_and_context_survives(ctx):
    g = __import__("conftest").load_golden("cfg2_n6000")
    n, d = g["Xr"].shape
    k = g["k"]
    prob = nat.Problem(n, d, k, g["group_ranges"], g["out_offsets"], g["out_ids"], route=nat.ROUTE_TENSOR)
    ids = np.empty(n * k, dtype=np.uint32)
    dists = np.empty(n * k, dtype=np.float32)
    ctx.prepare_base_vectors(g["Xr"], n, d, on_device=False)
    try:
        # the producer warp withholds all work: every consumer wait must run out
        ctx.set_device_wait_limit_ns(20_000_000)
        ctx.set_fault_injection(nat.INJECT_WITHHOLD_WORK)
        with pytest.raises(nat.UngxError) as e:
            ctx.generate(prob, ids, dists)
        assert e.value.status == nat.UNGX_ERR_TIMEOUT
        ctx.set_fault_injection(nat.INJECT_NONE)
        ctx.set_device_wait_limit_ns(4_000_000_000)
        ctx.generate(prob, ids, dists)
        assert_rows_match(ids, dists, g["ids"], g["dists"], k)
    finally:
        ctx.set_fault_injection(nat.INJECT_NONE)
        ctx.set_device_wait_limit_ns(4_000_000_000)
        ctx.release_base_vectors()
