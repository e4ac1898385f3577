"""Generates the golden fixtures under tests/golden/ from the REFERENCE's own code.

The reference has no cross-edge known-answer tests or fixtures of its own, so the
expected outputs here come from running the reference's compiled leaf sources
(TrieIndex, SearchQueue, FloatL2DistanceHandler) through oracle/ref_harness.cpp,
which restates UniNavGraph's grouping, reorder, LNG and CPU exact cross-edge scan
(UNG_CROSS_EDGE_IMPL=3).  Needs oracle/_ref/libungref.so, i.e. a build in a tree
that has the reference sources:

    make -C oracle ref REF=<reference checkout> && python tests/golden/make_golden.py

Each fixture stores how to regenerate its inputs (seeded generator parameters, or the
small input arrays themselves), a digest of the inputs, and the reference's outputs:
group order, reorder map, LNG out-neighbour sets, the cross-edge ids and distances of
every vector, and the additional edges (build_cross_edges_generate_additional, exact
variant) as (from, to) pairs in the reference's order.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from filtervectorcode_refactor_b200 import datasets  # noqa: E402

# name -> (config id, n, seed)
SEEDED = {
    "cfg1_n3000": (1, 3000, 11),
    "cfg2_n6000": (2, 6000, 12),
    "cfg3_n1500": (3, 1500, 13),
    "cfg4_n6000": (4, 6000, 14),
}


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def edge_case_inputs(seed: int = 5):
    """Small adversarial input: exact duplicate vectors (distance ties broken by id),
    an empty label set (the trie root becomes a group), singleton groups, targets
    smaller than k, groups without any superset, d not a multiple of 4 or 8."""
    rng = np.random.default_rng(seed)
    n, d = 700, 13
    X = rng.standard_normal((n, d)).astype(np.float32)
    X[100:140] = X[20]            # 40 copies of one vector
    X[300:310] = X[301]
    X[::7] = np.round(X[::7] * 4) / 4  # coarse values -> many equal distances
    sets = []
    for i in range(n):
        r = rng.random()
        if r < 0.03:
            sets.append([])
        elif r < 0.06:
            sets.append([int(rng.integers(50, 400))])     # mostly singleton groups
        else:
            u = int(rng.integers(1, 4))
            sets.append(sorted(rng.choice(np.arange(1, 7), size=u, replace=False).tolist()))
    sets[5] = [1, 2, 3, 4, 5, 6]  # a maximal set: group without supersets
    off = np.zeros(n + 1, dtype=np.uint64)
    off[1:] = np.cumsum([len(s) for s in sets])
    lab = np.array([x for s in sets for x in s], dtype=np.uint32)
    return X, off, lab


def make_one(ref, name, X, off, lab, k, extra):
    lg = ref.label_graph(off, lab)
    Xr = X[lg["new_to_old"]]
    ids, dists, pairs = ref.cross_exact(Xr, k, lg["group_first"], lg["out_offsets"], lg["out_ids"])
    add_from, add_to = ref.additional_edges(Xr, k, lg["group_first"], lg["out_offsets"], lg["out_ids"], ids)
    np.savez_compressed(
        os.path.join(HERE, name + ".npz"), k=k, input_digest=digest(X, off, lab), new_to_old=lg["new_to_old"],
        group_first=lg["group_first"], out_offsets=lg["out_offsets"], out_ids=lg["out_ids"], ids=ids,
        dists=dists, pairs=pairs, add_from=add_from, add_to=add_to, **extra)
    print(name, "n", X.shape[0], "d", X.shape[1], "G", lg["num_groups"], "E", len(lg["out_ids"]), "pairs", pairs,
          "additional", add_from.size)


def main():
    import oracle as O
    ref = O.reference()
    if ref is None:
        sys.exit("oracle/_ref/libungref.so is missing: run make -C oracle ref REF=<reference checkout>")
    for name, (cfg, n, seed) in SEEDED.items():
        c = datasets.make_config(cfg, seed=seed, n=n)
        make_one(ref, name, c["X"], c["label_offsets"], c["labels"], c["k"],
                 dict(cfg=cfg, n=n, seed=seed))
    X, off, lab = edge_case_inputs()
    for k in (8, 40):
        make_one(ref, f"edge_ties_k{k}", X, off, lab, k, dict(X=X, label_offsets=off, labels=lab))


if __name__ == "__main__":
    main()
