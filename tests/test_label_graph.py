"""The product's grouping / reorder / LNG (host C++ in libungx) against the reference goldens."""
import numpy as np
import pytest

import oracle as O
from filtervectorcode_refactor_b200 import _native as nat
from filtervectorcode_refactor_b200 import datasets


def test_label_graph_matches_golden(golden):
    lg = nat.LabelGraph(golden["label_offsets"], golden["labels"])
    G = golden["num_groups"]
    assert lg.num_groups == G
    assert np.array_equal(lg.new_to_old, golden["new_to_old"])
    assert np.array_equal(lg.group_ranges, golden["group_ranges"])
    assert O.lng_sets(lg.out_offsets, lg.out_ids, G) == O.lng_sets(golden["out_offsets"], golden["out_ids"], G)
    # in-neighbours: transpose of out, each list ascending (reference builds it serially)
    for t in range(1, G + 1):
        ins = lg.in_ids[lg.in_offsets[t]:lg.in_offsets[t + 1]]
        assert np.all(np.diff(ins.astype(np.int64)) > 0)
        for f in ins:
            assert t in lg.out_ids[lg.out_offsets[f]:lg.out_offsets[f + 1]]


def test_label_sets_are_sorted_sequences():
    off = np.array([0, 2, 4, 4, 5], dtype=np.uint64)
    lab = np.array([3, 1, 1, 3, 7], dtype=np.uint32)  # {3,1} and {1,3} are one group; empty set; {7}
    lg = nat.LabelGraph(off, lab)
    assert lg.num_groups == 3
    assert lg.new_to_old.tolist() == [0, 1, 2, 3]
    assert lg.set_labels.tolist() == [1, 3, 7]
    # empty set (group 2) has every other group as superset; minimal ones: {1,3} and {7}
    assert sorted(lg.out_ids[lg.out_offsets[2]:lg.out_offsets[3]].tolist()) == [1, 3]
    assert lg.out_offsets[2] - lg.out_offsets[1] == 0  # {1,3} has no strict superset


def test_label_graph_config2_shape():
    """Group statistics of the full config-2 label model (seed 0): 21,753 groups,
    5,316 singletons, 81,611 LNG edges, W = 1.549e10 pairs."""
    c = datasets.CONFIGS[2]
    off, lab = datasets.make_labels(c["n"], c["vocab"], c["umin"], c["umax"], c["zipf"], seed=0)
    lg = nat.LabelGraph(off, lab)
    sizes = np.diff(lg.group_ranges.reshape(-1, 2), axis=1)[1:, 0].astype(np.int64)
    assert lg.num_groups == 21753
    assert int((sizes == 1).sum()) == 5316
    assert len(lg.out_ids) == 81611
    W = 0
    for f in range(1, lg.num_groups + 1):
        outs = lg.out_ids[lg.out_offsets[f]:lg.out_offsets[f + 1]]
        W += int(sizes[f - 1]) * int(sizes[outs.astype(np.int64) - 1].sum())
    assert W == 15487870738 or abs(W - 1.549e10) / 1.549e10 < 1e-3


def test_label_graph_rejects_bad_offsets():
    off = np.array([0, 3, 2], dtype=np.uint64)
    lab = np.array([1, 2, 3], dtype=np.uint32)
    with pytest.raises(nat.UngxError):
        nat.LabelGraph(off, lab)


@pytest.mark.parametrize("vocab", [30, 100])
def test_label_graph_matches_reference_trie(vocab):
    """Both LNG paths against the reference's own TrieIndex build (oracle/_ref): label
    sets of up to 64 distinct labels take the mask scan, larger vocabularies the general
    inclusion test; empty label sets included."""
    ref = O.reference()
    if ref is None:
        pytest.skip("the reference harness (oracle/_ref) is not built")
    rng = np.random.default_rng(vocab)
    n = 20000
    sizes = rng.integers(0, 5, n)
    off = np.zeros(n + 1, dtype=np.uint64)
    off[1:] = np.cumsum(sizes)
    weights = 1.0 / np.arange(1, vocab + 1) ** 1.1
    weights /= weights.sum()
    lab = []
    for s in sizes:
        lab.extend(rng.choice(vocab, size=int(s), replace=False, p=weights).tolist())
    lab = np.array(lab, dtype=np.uint32)
    lg = nat.LabelGraph(off, lab)
    exp = ref.label_graph(off, lab)
    G = exp["num_groups"]
    assert np.array_equal(np.asarray(lg.new_to_old), exp["new_to_old"])
    assert np.array_equal(np.asarray(lg.group_ranges), exp["group_ranges"])
    got_sets = O.lng_sets(np.asarray(lg.out_offsets), np.asarray(lg.out_ids), G)
    exp_sets = O.lng_sets(exp["out_offsets"], exp["out_ids"], G)
    assert got_sets == exp_sets


def test_out_list_order_changes_only_row_order_of_additional_edges(golden):
    """The library returns each LNG out list in ascending group id; the reference keeps
    the order its trie search found them in (a breadth-first walk over hash-map children,
    uni_nav_graph_label_graph.cpp:103-206 and trie.cpp:78-143), which it never sorts.
    Cross edges depend only on the sets.  Additional edges follow the out-list order
    given to them: with either order the same (from, to) edges come out, and each
    point gets the same set, so a greedy search over the graph is unchanged."""
    from filtervectorcode_refactor_b200 import _native as nat
    g = golden
    G, k, n = g["num_groups"], g["k"], g["Xr"].shape[0]
    lg = nat.LabelGraph(g["label_offsets"], g["labels"])
    assert O.lng_sets(lg.out_offsets, lg.out_ids, G) == O.lng_sets(g["out_offsets"], g["out_ids"], G)
    for f in range(1, G + 1):
        row = lg.out_ids[lg.out_offsets[f]:lg.out_offsets[f + 1]]
        assert np.all(row[1:] > row[:-1])
    orc = O.oracle()
    ref_order = orc.additional_edges(g["Xr"], k, g["group_first"], g["out_offsets"], g["out_ids"], g["ids"])
    lib_order = orc.additional_edges(g["Xr"], k, g["group_first"], lg.out_offsets, lg.out_ids, g["ids"])
    assert np.array_equal(ref_order[0], g["add_from"]) and np.array_equal(ref_order[1], g["add_to"])
    pairs = lambda s, t: sorted(zip(s.tolist(), t.tolist()))
    assert pairs(*ref_order) == pairs(*lib_order)


@pytest.mark.parametrize("threads", [1, 3, 8])
def test_chunked_grouping_matches_serial_oracle(threads):
    """Above 2^18 points the grouping runs in parallel chunks merged in order; the
    group ids, reorder and LNG must equal a serial first-appearance pass, including
    empty label sets and groups whose first point sits late in a chunk."""
    from filtervectorcode_refactor_b200 import _native as nat
    rng = np.random.default_rng(threads)
    n = 300_000
    u = rng.integers(0, 4, size=n)                 # 0 = empty label set
    u[-5:] = 3                                     # new groups at the very end
    off = np.zeros(n + 1, dtype=np.uint64)
    off[1:] = np.cumsum(u)
    lab = np.concatenate([np.sort(rng.choice(12, size=c, replace=False)) + 1 for c in u]).astype(np.uint32)
    lab[-3:] = [20, 21, 22]                        # a label set only the last point has
    lg = nat.LabelGraph(off, lab, num_threads=threads)
    exp = O.oracle().label_graph(off, lab)
    G = exp["num_groups"]
    assert lg.num_groups == G
    assert np.array_equal(lg.new_to_old, exp["new_to_old"])
    assert np.array_equal(lg.group_ranges, exp["group_ranges"])
    assert O.lng_sets(lg.out_offsets, lg.out_ids, G) == O.lng_sets(exp["out_offsets"], exp["out_ids"], G)


def test_uninavgraph_mirror_host_steps(golden):
    """The host half of the UniNavGraph mirror: groups, reorder, the row -> group map
    and the LNG view, against the golden (the reference's grouping and trie)."""
    from filtervectorcode_refactor_b200.ung import UniNavGraph
    g = golden
    ung = UniNavGraph(num_cross_edges=g["k"])
    ung.build_trie_and_divide_groups(g["label_offsets"], g["labels"])
    ung.prepare_group_storages_graphs(g["X"])
    ung.build_label_nav_graph()
    assert np.array_equal(ung._new_to_old_vec_ids, g["new_to_old"])
    assert np.array_equal(ung._base, g["Xr"])
    gf = g["group_first"].astype(np.int64)
    exp = np.zeros(g["Xr"].shape[0], dtype=np.uint32)
    for f in range(1, g["num_groups"] + 1):
        exp[gf[f]:gf[f + 1]] = f
    assert np.array_equal(ung._new_vec_id_to_group_id, exp)
    for f in range(1, g["num_groups"] + 1):
        assert set(ung._label_nav_graph.out_neighbors(f).tolist()) == \
            set(g["out_ids"][g["out_offsets"][f]:g["out_offsets"][f + 1]].tolist())
