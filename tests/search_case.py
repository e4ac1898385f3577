"""Shared set-up of the filtered-search checks (benchmark configuration 5 at reduced
size): the configuration-2 index, its queries and the oracle-built graph.

The index graph of a point is, in the reference's order (UNG/codes/src/uni_nav_graph.cpp:
285-297 and the cross-edge merge): its intra-group edges, its cross edges in queue order,
then its additional edges.  The intra-group edges come from the exact kNN seeding
(candidate K 64, degree 32); the cross and additional edges from the exact build."""
import numpy as np

import oracle as O
from filtervectorcode_refactor_b200 import _native as nat
from filtervectorcode_refactor_b200 import datasets

KNN_K, KNN_DEGREE = 64, 32


def make_case(n: int, nq: int, seed: int) -> dict:
    c = datasets.make_config(2, seed=seed, n=n)
    qc = datasets.make_queries(seed=seed, nq=nq)
    lg = nat.LabelGraph(c["label_offsets"], c["labels"])
    gf = np.concatenate([[0], lg.group_ranges[2::2], [lg.group_ranges[-1]]]).astype(np.uint32)
    to, ti, mo, mi = O.query_groups(lg.set_offsets, lg.set_labels, qc["label_offsets"], qc["labels"])
    grp_of = np.repeat(np.arange(1, lg.num_groups + 1, dtype=np.int64), np.diff(gf.astype(np.int64))[1:])
    return dict(n=n, k=c["k"], Xr=np.ascontiguousarray(c["X"][lg.new_to_old]), group_ranges=lg.group_ranges,
                group_first=gf, group_of=grp_of, out_offsets=lg.out_offsets, out_ids=lg.out_ids,
                num_groups=lg.num_groups, Q=qc["Q"], L=qc["L"], K=qc["K"], E=qc["num_entry_points"],
                target_offsets=to, target_ids=ti, min_offsets=mo, min_ids=mi, seed=seed)


def knn_config():
    return nat.exact_knn_default_config(KNN_K, KNN_DEGREE)


def intra_csr(graph_rows: np.ndarray, case: dict):
    """[degree, local ids ...] rows -> CSR over global ids."""
    deg = graph_rows[:, 0].astype(np.int64)
    off = np.zeros(case["n"] + 1, dtype=np.uint64)
    off[1:] = np.cumsum(deg)
    mask = np.arange(graph_rows.shape[1] - 1)[None, :] < deg[:, None]
    glob = graph_rows[:, 1:].astype(np.int64) + case["group_first"][case["group_of"]][:, None]
    return off, glob[mask].astype(np.uint32)


def assemble_graph(n: int, intra_off, intra_cols, cross_ids: np.ndarray, add_from, add_to):
    """Per point: intra-group edges, cross edges in queue order (empty slots dropped),
    additional edges in list order, as CSR (offsets uint64 [n+1], columns uint32)."""
    k = cross_ids.size // n
    cross = cross_ids.reshape(n, k)
    valid = cross != 0xFFFFFFFF
    intra_pt = np.repeat(np.arange(n, dtype=np.int64), np.diff(intra_off.astype(np.int64)))
    cross_pt = np.nonzero(valid)[0].astype(np.int64)
    keys = np.concatenate([3 * intra_pt, 3 * cross_pt + 1, 3 * add_from.astype(np.int64) + 2])
    vals = np.concatenate([intra_cols, cross[valid], add_to]).astype(np.uint32)
    order = np.argsort(keys, kind="stable")
    off = np.zeros(n + 1, dtype=np.uint64)
    off[1:] = np.cumsum(np.bincount(keys // 3, minlength=n))
    return off, vals[order]


def oracle_graph(case: dict, intra_rows=None, lib=None):
    """The whole index graph from the CPU checkers: CSR offsets, columns, and the
    groups' entry points (local index per group 0..G, 0 unused).  Cross and additional
    edges come from ``lib`` (the C restatement by default; ``oracle.reference()`` for the
    reference's own compiled code).  ``intra_rows`` replaces the oracle's kNN seeding
    with given [degree, local ids ...] rows (entry points then 0, as the seeding writes)."""
    lib = lib or O.oracle()
    if intra_rows is None:
        cfg = knn_config()
        intra_rows, entry = O.oracle().exact_knn_graph(case["Xr"], case["group_ranges"][2:], cfg.candidate_k,
                                                       cfg.final_degree, cfg.head_keep, cfg.anchor_tail,
                                                       cfg.anchor_slots, cfg.bidir_anchor, cfg.graph_stride)
    else:
        entry = np.zeros(case["num_groups"], dtype=np.uint32)
    i_off, i_cols = intra_csr(intra_rows, case)
    n, k = case["n"], case["k"]
    ids, _, _ = lib.cross_exact(case["Xr"], k, case["group_first"], case["out_offsets"], case["out_ids"])
    src, dst = lib.additional_edges(case["Xr"], k, case["group_first"], case["out_offsets"], case["out_ids"], ids)
    off, cols = assemble_graph(n, i_off, i_cols, ids, src, dst)
    group_entry = np.zeros(case["num_groups"] + 1, dtype=np.uint32)
    group_entry[1:] = entry
    return off, cols, group_entry


def search_recall(case: dict, offsets, cols, group_entry, truth=None):
    """Greedy search of every query (oracle restatement) and recall@K against the
    filtered brute-force truth (computed unless given): (recall, result ids, truth ids)."""
    orc = O.oracle()
    eo, ei = O.entry_points(case["group_first"], group_entry, case["min_offsets"], case["min_ids"], case["E"],
                            seed=case["seed"])
    res, _ = orc.ung_search(case["Xr"], offsets, cols, case["Q"], eo, ei, case["L"], case["K"])
    if truth is None:
        truth, _ = orc.filtered_scan(case["Xr"], case["group_first"], case["Q"], case["target_offsets"],
                                     case["target_ids"], case["K"])
    return O.recall_at_k(res, truth), res, truth
