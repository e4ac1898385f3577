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
