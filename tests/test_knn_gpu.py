"""Exact kNN graph seeding on the device (ungx_exact_knn_graph_device) against the
reference's own GPU kernel and the oracle restatement, bit for bit: every row (degree,
local ids in the head / anchor / tail layout, padding) and the entry points, over group
sizes from 1 to above the 64-row block, dimensions that are and are not multiples of
4 / 32 / 128, data with exact duplicates (ties broken by local id), and several layout
configurations.

The pin: oracle/_ref/libungref_knn.so is the reference's tagore_graph_builder.cu
compiled where it lies (with its --use_fast_math), run through its public batch entry
point on the exact route (batched_exact_knn_graph_kernel); the device rows must equal
its rows, and the C restatement must too."""
import numpy as np
import pytest

import oracle as O
from filtervectorcode_refactor_b200 import _native as nat

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SIZES = [1, 2, 5, 33, 64, 65, 100, 300, 1100]


@pytest.fixture(scope="module")
def ctx():
    c = nat.Context(0)
    yield c
    c.close()


def make_groups(d, seed):
    rng = np.random.default_rng(seed)
    n = sum(SIZES) + 7
    X = rng.standard_normal((n, d)).astype(np.float32)
    X[200:230] = X[205]                        # duplicates: equal distances, order by id
    X[::11] = np.round(X[::11] * 2) / 2        # coarse rows: more equal distances
    ranges, at = [], 3                         # a few leading rows outside every group
    for s in SIZES:
        ranges += [at, at + s]
        at += s
    return X, np.array(ranges, dtype=np.uint32)


CONFIGS = {
    "default": lambda: nat.exact_knn_default_config(64, 32),
    "small_k": lambda: _cfg(20, 16, 10, 1, 3, 1, 17),
    "no_anchor": lambda: _cfg(40, 24, 24, 0, 0, 0, 30),
    "stride_k": lambda: _cfg(64, 32, 24, 1, 0, 0, 64),
}


def _cfg(k, deg, head, tail, slots, bidir, stride):
    c = nat.ExactKnnConfig()
    c.candidate_k, c.final_degree, c.head_keep, c.anchor_tail = k, deg, head, tail
    c.anchor_slots, c.bidir_anchor, c.graph_stride = slots, bidir, stride
    return c


ROUTES = {"tensor": nat.ROUTE_TENSOR, "exact": nat.ROUTE_EXACT}


# dims: one to three 128-dim segments per partial; 4-, 8- and 16-byte staging copies
DIMS = [13, 96, 98, 128, 200, 259, 262, 300]


@pytest.mark.parametrize("d", DIMS)
@pytest.mark.parametrize("name", list(CONFIGS))
@pytest.mark.parametrize("route", list(ROUTES))
def test_exact_knn_graph_matches_oracle(ctx, d, name, route):
    run_against_oracle(ctx, d, name, ROUTES[route])


def run_against_oracle(ctx, d, name, route=nat.ROUTE_AUTO):
    """Device rows of one case, checked against the C restatement; returns the case."""
    X, ranges = make_groups(d, seed=d)
    cfg = CONFIGS[name]()
    cfg.route = route
    pts = int(np.sum(ranges[1::2].astype(np.int64) - ranges[0::2]))
    ctx.prepare_base_vectors(X, X.shape[0], d, on_device=False)
    d_graph = torch.full((pts, cfg.graph_stride), 7, dtype=torch.int32, device="cuda")
    d_entry = torch.full((ranges.size // 2,), 9, dtype=torch.int32, device="cuda")
    ctx.exact_knn_graph_device(ranges, cfg, d_graph.data_ptr(), d_entry.data_ptr())
    if route == nat.ROUTE_TENSOR:
        print(f"kNN tensor route d={d} {name}: {ctx.knn_rejected_rows()} rows rejected")
    ctx.release_base_vectors()
    got = d_graph.cpu().numpy().view(np.uint32)
    exp, exp_entry = O.oracle().exact_knn_graph(X, ranges, cfg.candidate_k, cfg.final_degree, cfg.head_keep,
                                                cfg.anchor_tail, cfg.anchor_slots, cfg.bidir_anchor,
                                                cfg.graph_stride)
    assert np.array_equal(d_entry.cpu().numpy().view(np.uint32), exp_entry)
    bad = np.nonzero(np.any(got != exp, axis=1))[0]
    assert bad.size == 0, f"{bad.size} rows differ; first {bad[0]}: got {got[bad[0]].tolist()} " \
                          f"expected {exp[bad[0]].tolist()}"
    return X, ranges, cfg, got


@pytest.mark.parametrize("d", DIMS)
@pytest.mark.parametrize("name", list(CONFIGS))
@pytest.mark.parametrize("route", list(ROUTES))
def test_exact_knn_graph_matches_reference_kernel(ctx, d, name, route):
    """The device rows (both routes) and the oracle's equal the reference's own GPU kernel's rows."""
    ref = O.reference_knn()
    if ref is None:
        pytest.skip("oracle/_ref/libungref_knn.so is not built (the reference tree was absent at build time)")
    X, ranges, cfg, got = run_against_oracle(ctx, d, name, ROUTES[route])
    exp, exp_entry = ref.exact_knn_graph(X, ranges, cfg.candidate_k, cfg.final_degree, cfg.head_keep,
                                         cfg.anchor_tail, cfg.anchor_slots, cfg.bidir_anchor, cfg.graph_stride)
    assert np.all(exp_entry == 0)
    bad = np.nonzero(np.any(got != exp, axis=1))[0]
    assert bad.size == 0, f"{bad.size} rows differ from the reference kernel; first {bad[0]}: " \
                          f"got {got[bad[0]].tolist()} reference {exp[bad[0]].tolist()}"


def test_dimension_limit_is_refused(ctx):
    X = np.zeros((10, 400), dtype=np.float32)
    ctx.prepare_base_vectors(X, 10, 400, on_device=False)
    cfg = nat.exact_knn_default_config(64, 32)
    d_graph = torch.zeros((10, 33), dtype=torch.int32, device="cuda")
    with pytest.raises(nat.UngxError):
        ctx.exact_knn_graph_device(np.array([0, 10], dtype=np.uint32), cfg, d_graph.data_ptr())
    ctx.release_base_vectors()


# The two-phase path in many batches (every group in its own batch) and the fused
# kernel (taken for groups above the two-phase limit) give the same rows.
PATHS = {"batched": ("UNGX_KNN_BATCH_ENTRIES", "20000"), "fused": ("UNGX_KNN_DIST_MAX_N", "0")}


@pytest.mark.parametrize("d", [13, 128])
@pytest.mark.parametrize("name", ["default", "small_k"])
@pytest.mark.parametrize("path", list(PATHS))
def test_exact_knn_paths_match_oracle(ctx, monkeypatch, d, name, path):
    monkeypatch.setenv(*PATHS[path])
    run_against_oracle(ctx, d, name, nat.ROUTE_EXACT)


@pytest.mark.parametrize("d", [64, 128, 300])
def test_tensor_route_large_groups_match_oracle(ctx, d):
    """Groups of 2,000 and 9,000 points (above the exact route's matrix limit) on the tensor
    route: rows equal the oracle's; the certificate clears nearly every row."""
    rng = np.random.default_rng(77 + d)
    sizes = [2000, 9000, 300]
    X = rng.standard_normal((sum(sizes), d)).astype(np.float32)
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    ranges, at = [], 0
    for sz in sizes:
        ranges += [at, at + sz]
        at += sz
    ranges = np.array(ranges, dtype=np.uint32)
    cfg = nat.exact_knn_default_config(64, 32)
    pts = X.shape[0]
    ctx.prepare_base_vectors(X, pts, d, on_device=False)
    d_graph = torch.zeros((pts, cfg.graph_stride), dtype=torch.int32, device="cuda")
    ctx.exact_knn_graph_device(ranges, cfg, d_graph.data_ptr())
    rejected = ctx.knn_rejected_rows()
    ctx.release_base_vectors()
    got = d_graph.cpu().numpy().view(np.uint32)
    exp, _ = O.oracle().exact_knn_graph(X, ranges, cfg.candidate_k, cfg.final_degree, cfg.head_keep,
                                        cfg.anchor_tail, cfg.anchor_slots, cfg.bidir_anchor, cfg.graph_stride)
    bad = np.nonzero(np.any(got != exp, axis=1))[0]
    assert bad.size == 0, f"{bad.size} rows differ; first {bad[0]}"
    print(f"kNN tensor route, groups {sizes}, d={d}: {rejected} of {pts} rows rejected")
    assert rejected <= 0.03 * pts


def test_tensor_route_many_groups_equal_exact_route(ctx):
    """Thousands of groups of 65..400 points and one of 70,000 (above 2^16, so local ids
    and rejected-row slots need more than 16 bits): the tensor route's rows, with the
    rejected rows grouped and recomputed on the device, equal the exact route's rows."""
    rng = np.random.default_rng(2024)
    sizes = list(rng.integers(65, 401, size=2500)) + [70000] + list(rng.integers(65, 401, size=500))
    d = 16
    n = int(sum(sizes))
    X = rng.standard_normal((n, d)).astype(np.float32)
    X[:n // 3] = np.round(X[:n // 3] * 4) / 4          # coarse values: equal distances, ties by id
    ranges, at = [], 0
    for sz in sizes:
        ranges += [at, at + int(sz)]
        at += int(sz)
    ranges = np.array(ranges, dtype=np.uint32)
    ctx.prepare_base_vectors(X, n, d, on_device=False)
    rows = {}
    try:
        for name, route in ROUTES.items():
            cfg = nat.exact_knn_default_config(64, 32)
            cfg.route = route
            g = torch.full((n, cfg.graph_stride), 7, dtype=torch.int32, device="cuda")
            e = torch.full((len(sizes),), 9, dtype=torch.int32, device="cuda")
            ctx.exact_knn_graph_device(ranges, cfg, g.data_ptr(), e.data_ptr())
            rows[name] = (g.cpu().numpy(), e.cpu().numpy())
            if route == nat.ROUTE_TENSOR:
                rejected = ctx.knn_rejected_rows()
    finally:
        ctx.release_base_vectors()
    assert np.array_equal(rows["tensor"][1], rows["exact"][1])
    bad = np.nonzero(np.any(rows["tensor"][0] != rows["exact"][0], axis=1))[0]
    assert bad.size == 0, f"{bad.size} rows differ; first {bad[0]}"
    print(f"many groups: {rejected} of {n} rows rejected")
    assert rejected > 0  # the fallback path ran
