"""The filtered-search checkers (benchmark configuration 5) on the CPU:

* the greedy search restatement (orc_ung_search) returns what iterate_to_fixed_point
  over the reference's own SearchQueue and distance returns (ungref_ung_search);
* the filtered brute-force truth (orc_filtered_scan) equals FilteredScan's queue order
  over the reference's own SearchQueue, ids and distance bits;
* on a graph that links every point to all points of the groups containing its label
  set, a queue that holds every reachable point returns exactly the truth: the search
  never leaves the containment targets and loses nothing;
* query groups: containment targets include the query's set, entry groups are the
  minimal ones among them."""
import numpy as np
import pytest

import oracle as O
from search_case import make_case, oracle_graph, search_recall


@pytest.fixture(scope="module")
def case():
    return make_case(4000, 160, seed=11)


@pytest.fixture(scope="module")
def graph(case):
    return oracle_graph(case)


def test_search_matches_reference_queue(case, graph):
    ref = O.reference()
    if ref is None:
        pytest.skip("reference build (oracle/_ref) absent")
    off, cols, ge = graph
    eo, ei = O.entry_points(case["group_first"], ge, case["min_offsets"], case["min_ids"], case["E"], seed=1)
    for L, K in [(case["L"], case["K"]), (12, 10), (40, 1)]:
        got, cmps = O.oracle().ung_search(case["Xr"], off, cols, case["Q"], eo, ei, L, K)
        exp = ref.ung_search(case["Xr"], off, cols, case["Q"], eo, ei, L, K)
        assert np.array_equal(got, exp), f"L={L} K={K}"
        assert np.all(cmps >= np.diff(eo).astype(np.uint32))


def test_filtered_scan_matches_reference(case):
    ref = O.reference()
    if ref is None:
        pytest.skip("reference build (oracle/_ref) absent")
    for K in (1, 10, 37):
        gi, gd = O.oracle().filtered_scan(case["Xr"], case["group_first"], case["Q"], case["target_offsets"],
                                          case["target_ids"], K)
        ri, rd = ref.filtered_scan(case["Xr"], case["group_first"], case["Q"], case["target_offsets"],
                                   case["target_ids"], K)
        assert np.array_equal(gi, ri)
        assert np.array_equal(gd.view(np.uint32), rd.view(np.uint32))


def test_query_groups_are_containment_and_minimal(case):
    from filtervectorcode_refactor_b200 import _native as nat
    from filtervectorcode_refactor_b200 import datasets
    c = datasets.make_config(2, seed=case["seed"], n=case["n"])
    qc = datasets.make_queries(seed=case["seed"], nq=case["Q"].shape[0])
    lg = nat.LabelGraph(c["label_offsets"], c["labels"])
    sets = [set(lg.set_labels[lg.set_offsets[g]:lg.set_offsets[g + 1]].tolist()) for g in range(lg.num_groups + 1)]
    for q in range(qc["nq"]):
        qs = set(qc["labels"][qc["label_offsets"][q]:qc["label_offsets"][q + 1]].tolist())
        tg = case["target_ids"][case["target_offsets"][q]:case["target_offsets"][q + 1]].tolist()
        mg = case["min_ids"][case["min_offsets"][q]:case["min_offsets"][q + 1]].tolist()
        assert tg == [g for g in range(1, lg.num_groups + 1) if qs <= sets[g]]
        assert set(mg) <= set(tg)
        for g in tg:
            assert any(sets[m] <= sets[g] for m in mg)
        for m in mg:
            assert not any(sets[o] < sets[m] for o in tg)


def test_closure_graph_search_equals_truth():
    c = make_case(700, 64, seed=3)
    G, gf = c["num_groups"], c["group_first"]
    from filtervectorcode_refactor_b200 import _native as nat
    from filtervectorcode_refactor_b200 import datasets
    d = datasets.make_config(2, seed=3, n=700)
    lg = nat.LabelGraph(d["label_offsets"], d["labels"])
    sets = [set(lg.set_labels[lg.set_offsets[g]:lg.set_offsets[g + 1]].tolist()) for g in range(G + 1)]
    rows = []
    for v in range(c["n"]):
        s = sets[int(c["group_of"][v])]
        r = []
        for g in range(1, G + 1):
            if s <= sets[g]:
                r += [x for x in range(int(gf[g]), int(gf[g + 1])) if x != v]
        rows.append(r)
    off = np.zeros(c["n"] + 1, dtype=np.uint64)
    off[1:] = np.cumsum([len(r) for r in rows])
    cols = np.array([x for r in rows for x in r], dtype=np.uint32)
    c["L"] = c["n"]
    recall, res, gt = search_recall(c, off, cols, np.zeros(G + 1, dtype=np.uint32))
    assert np.array_equal(res, gt)
    assert recall == 1.0


def test_recall_counts_truth_slots():
    res = np.array([[1, 2, 3], [4, 5, 6]], dtype=np.uint32)
    gt = np.array([[3, 2, 9], [4, 0xFFFFFFFF, 0xFFFFFFFF]], dtype=np.uint32)
    assert O.recall_at_k(res, gt) == pytest.approx(3 / 4)


def test_assemble_graph_order():
    """Per point: intra edges, cross edges up to the first empty slot, additional edges
    in list order; points without edges get empty rows."""
    from search_case import assemble_graph
    S = 0xFFFFFFFF
    n, k = 4, 3
    intra_off = np.array([0, 2, 2, 3, 3], dtype=np.uint64)
    intra_cols = np.array([7, 8, 9], dtype=np.uint32)
    cross = np.array([[1, 2, S], [S, S, S], [3, S, S], [4, 5, 6]], dtype=np.uint32).ravel()
    add_from = np.array([3, 0, 3], dtype=np.uint32)
    add_to = np.array([10, 11, 12], dtype=np.uint32)
    off, cols = assemble_graph(n, intra_off, intra_cols, cross, add_from, add_to)
    rows = [cols[off[v]:off[v + 1]].tolist() for v in range(n)]
    assert rows == [[7, 8, 1, 2, 11], [], [9, 3], [4, 5, 6, 10, 12]]


def test_search_ignores_column_order_within_rows(case, graph):
    """One expansion inserts all of a node's unvisited neighbours before the next one
    starts, and the bounded queue keeps the best L of what it has seen, so the result
    does not depend on the order of a row's columns (e.g. of its additional edges)."""
    off, cols, ge = graph
    rev = cols.copy()
    for v in range(case["n"]):
        rev[off[v]:off[v + 1]] = cols[off[v]:off[v + 1]][::-1]
    r1, res1, _ = search_recall(case, off, cols, ge)
    r2, res2, _ = search_recall(case, off, rev, ge)
    assert np.array_equal(res1, res2) and r1 == r2
