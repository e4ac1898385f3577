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


def oracle_graph(case: dict):
    """The whole index graph from the CPU oracle: CSR offsets, columns, and the groups'
    entry points (local index per group 0..G, 0 unused)."""
    orc = O.oracle()
    cfg = knn_config()
    rows, entry = orc.exact_knn_graph(case["Xr"], case["group_ranges"][2:], cfg.candidate_k, cfg.final_degree,
                                      cfg.head_keep, cfg.anchor_tail, cfg.anchor_slots, cfg.bidir_anchor,
                                      cfg.graph_stride)
    i_off, i_cols = intra_csr(rows, case)
    n, k = case["n"], case["k"]
    ids, _, _ = orc.cross_exact(case["Xr"], k, case["group_first"], case["out_offsets"], case["out_ids"])
    src, dst = orc.additional_edges(case["Xr"], k, case["group_first"], case["out_offsets"], case["out_ids"], ids)
    cross = ids.reshape(n, k)
    order = np.argsort(src, kind="stable")
    a_off = np.zeros(n + 1, dtype=np.int64)
    a_off[1:] = np.cumsum(np.bincount(src, minlength=n))
    a_dst = dst[order]
    rows_out = []
    for v in range(n):
        r = i_cols[i_off[v]:i_off[v + 1]].tolist()
        r += [x for x in cross[v].tolist() if x != 0xFFFFFFFF]
        r += a_dst[a_off[v]:a_off[v + 1]].tolist()
        rows_out.append(r)
    off = np.zeros(n + 1, dtype=np.uint64)
    off[1:] = np.cumsum([len(r) for r in rows_out])
    cols = np.fromiter((x for r in rows_out for x in r), dtype=np.uint32, count=int(off[-1]))
    group_entry = np.zeros(case["num_groups"] + 1, dtype=np.uint32)
    group_entry[1:] = entry
    return off, cols, group_entry


def search_recall(case: dict, offsets, cols, group_entry):
    """Greedy search of every query (oracle restatement) and recall@K against the
    filtered brute-force truth: (recall, result ids, truth ids)."""
    orc = O.oracle()
    eo, ei = O.entry_points(case["group_first"], group_entry, case["min_offsets"], case["min_ids"], case["E"],
                            seed=case["seed"])
    res, _ = orc.ung_search(case["Xr"], offsets, cols, case["Q"], eo, ei, case["L"], case["K"])
    gt, _ = orc.filtered_scan(case["Xr"], case["group_first"], case["Q"], case["target_offsets"],
                              case["target_ids"], case["K"])
    return O.recall_at_k(res, gt), res, gt
