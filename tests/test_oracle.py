"""Pins the CPU oracle: the plain-C restatement must reproduce the reference's own
outputs (golden fixtures made by the reference's compiled code) bit for bit."""
import numpy as np
import pytest

import oracle as O


def test_oracle_label_graph_matches_golden(golden):
    o = O.oracle().label_graph(golden["label_offsets"], golden["labels"])
    G = golden["num_groups"]
    assert o["num_groups"] == G
    assert np.array_equal(o["new_to_old"], golden["new_to_old"])
    assert np.array_equal(o["group_first"], golden["group_first"])
    assert O.lng_sets(o["out_offsets"], o["out_ids"], G) == O.lng_sets(golden["out_offsets"], golden["out_ids"], G)


def test_oracle_cross_exact_matches_golden(golden):
    ids, dists, pairs = O.oracle().cross_exact(golden["Xr"], golden["k"], golden["group_first"],
                                               golden["out_offsets"], golden["out_ids"])
    assert pairs == int(golden["pairs"])
    assert np.array_equal(ids, golden["ids"])
    assert np.array_equal(dists.view(np.uint32), golden["dists"].view(np.uint32))


@pytest.mark.parametrize("d", [1, 3, 4, 5, 7, 8, 12, 13, 96, 99, 128, 131, 960])
def test_oracle_l2_bitexact_vs_reference(d):
    ref = O.reference()
    if ref is None:
        pytest.skip("reference build (oracle/_ref) not present on this machine")
    orc = O.oracle()
    rng = np.random.default_rng(d)
    for _ in range(64):
        a = rng.standard_normal(d).astype(np.float32)
        b = rng.standard_normal(d).astype(np.float32) * np.float32(rng.random())
        r, o = np.float32(ref.l2(a, b)), np.float32(orc.l2(a, b))
        assert r.view(np.uint32) == o.view(np.uint32)


def test_reference_harness_reproduces_golden(golden):
    ref = O.reference()
    if ref is None:
        pytest.skip("reference build (oracle/_ref) not present on this machine")
    ids, dists, _ = ref.cross_exact(golden["Xr"], golden["k"], golden["group_first"], golden["out_offsets"],
                                    golden["out_ids"])
    assert np.array_equal(ids, golden["ids"])


def test_oracle_additional_edges_match_golden(golden):
    """Additional edges (the exact variant of build_cross_edges_generate_additional):
    the C restatement reproduces the reference harness's (from, to) list in order."""
    src, dst = O.oracle().additional_edges(golden["Xr"], golden["k"], golden["group_first"], golden["out_offsets"],
                                           golden["out_ids"], golden["ids"])
    assert np.array_equal(src, golden["add_from"])
    assert np.array_equal(dst, golden["add_to"])


def test_reference_harness_reproduces_golden_additional_edges(golden):
    ref = O.reference()
    if ref is None:
        pytest.skip("reference build (oracle/_ref) not present on this machine")
    src, dst = ref.additional_edges(golden["Xr"], golden["k"], golden["group_first"], golden["out_offsets"],
                                    golden["out_ids"], golden["ids"])
    assert np.array_equal(src, golden["add_from"]) and np.array_equal(dst, golden["add_to"])


@pytest.mark.parametrize("d", [3, 13, 259])
def test_oracle_additional_edges_match_reference_at_ragged_dims(d):
    """The C restatement's cross edges and additional edges equal the reference harness's
    at dimensions with 8-wide and 4-wide tails (the oracle the device's ragged-dimension
    additional-edge test compares with), on a configuration-2 label structure of 3,000
    points with coarse, tie-heavy values."""
    ref = O.reference()
    if ref is None:
        pytest.skip("reference build (oracle/_ref) not present on this machine")
    from filtervectorcode_refactor_b200 import _native as nat
    from filtervectorcode_refactor_b200 import datasets
    c = datasets.make_config(2, seed=7 + d, n=3000)
    lg = nat.LabelGraph(c["label_offsets"], c["labels"])
    gf = np.concatenate([[0], lg.group_ranges[2::2], [lg.group_ranges[-1]]]).astype(np.uint32)
    X = np.random.default_rng(d).integers(-40, 40, size=(3000, d)).astype(np.float32) / 8
    k = c["k"]
    ids, dists, _ = O.oracle().cross_exact(X, k, gf, lg.out_offsets, lg.out_ids)
    rids, rdists, _ = ref.cross_exact(X, k, gf, lg.out_offsets, lg.out_ids)
    assert np.array_equal(ids, rids)
    assert np.array_equal(dists.view(np.uint32), rdists.view(np.uint32))
    src, dst = O.oracle().additional_edges(X, k, gf, lg.out_offsets, lg.out_ids, ids)
    rsrc, rdst = ref.additional_edges(X, k, gf, lg.out_offsets, lg.out_ids, rids)
    assert src.size > 0
    assert np.array_equal(src, rsrc) and np.array_equal(dst, rdst)


def test_planted_mistake_is_caught(golden):
    """A mistake planted in the oracle's output (on the CPU) must fail the comparison
    the GPU tests use."""
    from parity import assert_rows_match
    ids = golden["ids"].copy()
    dists = golden["dists"].copy()
    k = golden["k"]
    row = int(np.argmax(ids.reshape(-1, k)[:, 0] != 0xFFFFFFFF))
    ids[row * k] ^= 1
    with pytest.raises(AssertionError):
        assert_rows_match(ids, dists, golden["ids"], golden["dists"], k)


@pytest.mark.parametrize("name", __import__("adversarial").CASES)
def test_oracle_matches_reference_on_certificate_edge_cases(name):
    """The certificate's adversarial inputs (huge norm spans, fp16-subnormal operands,
    an element beyond fp16's range with +inf distances, a large offset, ties): the C
    restatement equals the reference's own compiled exact scan on every row."""
    from adversarial import make_case
    X, k, first, ranges, off, ids = make_case(name)
    o_ids, o_d, o_pairs = O.oracle().cross_exact(X, k, first, off, ids)
    assert o_pairs > 0
    ref = O.reference()
    if ref is None:
        pytest.skip("reference build (oracle/_ref) not present on this machine")
    r_ids, r_d, r_pairs = ref.cross_exact(X, k, first, off, ids)
    assert r_pairs == o_pairs
    assert np.array_equal(r_ids, o_ids)
    assert np.array_equal(r_d.view(np.uint32), o_d.view(np.uint32))


def test_row_property_checkers_agree_and_catch_mistakes(golden):
    """The vectorised size-independent row checker accepts every golden row, as the
    per-row one does, and rejects planted mistakes (an unsorted row, an id outside the
    row's out-groups, a missing edge)."""
    from parity import check_row_properties, check_row_properties_fast
    k = golden["k"]
    ids, d = golden["ids"].copy(), golden["dists"].copy()
    n = ids.size // k
    args = (k, golden["group_ranges"], golden["out_offsets"], golden["out_ids"])
    assert check_row_properties_fast(ids, d, *args, np.arange(n)) == n
    check_row_properties(ids, d, *args, np.arange(min(n, 300)))
    full = np.nonzero(np.all(ids.reshape(-1, k) != 0xFFFFFFFF, axis=1))[0]
    r = int(full[0])
    for plant in ("swap", "foreign", "missing"):
        i2, d2 = ids.copy().reshape(-1, k), d.copy().reshape(-1, k)
        if plant == "swap":
            i2[r, [0, 1]] = i2[r, [1, 0]]
            d2[r, [0, 1]] = d2[r, [1, 0]]
            if d2[r, 0] == d2[r, 1]:
                continue
        elif plant == "foreign":
            i2[r, k - 1] = r  # the row itself: never in its own out-groups
        else:
            i2[r, k - 1] = 0xFFFFFFFF
            d2[r, k - 1] = np.inf
        with pytest.raises(AssertionError):
            check_row_properties_fast(i2.ravel(), d2.ravel(), *args, np.array([r]))


def test_reference_knn_library_loads():
    """The reference's GPU kNN seeding checker links completely (it runs only in GPU tests)."""
    if not __import__("os").path.exists(O.REF_KNN_SO):
        pytest.skip("oracle/_ref/libungref_knn.so not built on this machine")
    assert O.reference_knn() is not None
