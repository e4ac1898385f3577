"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU checkers.

* ``_build/libungx_oracle.so`` -- the plain-C restatement (ungx_oracle.c), always built.
* ``_ref/libungref.so``        -- the reference's own leaf sources (TrieIndex, SearchQueue,
  FloatL2DistanceHandler) compiled where they lie, plus ref_harness.cpp; present
  only where the reference tree was available at build time.
* ``_ref/libungref_knn.so``    -- the reference's GPU exact kNN seeding
  (tagore_graph_builder.cu compiled where it lies) behind knn_ref_harness.cpp; it runs
  on the GPU, so only GPU tests call it.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_float, c_int, c_uint8, c_uint32, c_uint64, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libungx_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libungref.so")
REF_KNN_SO = os.path.join(HERE, "_ref", "libungref_knn.so")

# FloatL2DistanceHandler's rounding in the reference's release build: the 8-lane
# loop rounds mul and add separately, the tails are fused (bit 1).
L2_REFERENCE_BUILD = 2


def _p(a):
    return None if a is None else a.ctypes.data


class _Lib:
    def __init__(self, path: str, prefix: str):
        self.lib = ctypes.CDLL(path)
        self.prefix = prefix
        L, P = self.lib, prefix
        getattr(L, f"{P}label_graph_build").restype = c_void_p
        getattr(L, f"{P}label_graph_build").argtypes = [c_uint32, c_void_p, c_void_p]
        getattr(L, f"{P}num_groups").restype = c_uint32
        getattr(L, f"{P}num_groups").argtypes = [c_void_p]
        getattr(L, f"{P}copy_groups").argtypes = [c_void_p, c_void_p, c_void_p]
        getattr(L, f"{P}lng_nnz").restype = c_uint64
        getattr(L, f"{P}lng_nnz").argtypes = [c_void_p]
        getattr(L, f"{P}copy_lng_out").argtypes = [c_void_p, c_void_p, c_void_p]
        getattr(L, f"{P}label_graph_free").argtypes = [c_void_p]

    def label_graph(self, label_offsets: np.ndarray, labels: np.ndarray) -> dict:
        P = self.prefix
        label_offsets = np.ascontiguousarray(label_offsets, dtype=np.uint64)
        labels = np.ascontiguousarray(labels, dtype=np.uint32)
        n = label_offsets.shape[0] - 1
        h = getattr(self.lib, f"{P}label_graph_build")(n, _p(label_offsets), _p(labels) if labels.size else None)
        try:
            G = getattr(self.lib, f"{P}num_groups")(h)
            new_to_old = np.empty(n, dtype=np.uint32)
            first = np.empty(G + 2, dtype=np.uint32)
            getattr(self.lib, f"{P}copy_groups")(h, _p(new_to_old), _p(first))
            nnz = getattr(self.lib, f"{P}lng_nnz")(h)
            off = np.empty(G + 2, dtype=np.uint64)
            ids = np.empty(max(nnz, 1), dtype=np.uint32)
            getattr(self.lib, f"{P}copy_lng_out")(h, _p(off), _p(ids))
        finally:
            getattr(self.lib, f"{P}label_graph_free")(h)
        ranges = np.zeros(2 * (G + 1), dtype=np.uint32)
        ranges[2::2] = first[1:G + 1]
        ranges[3::2] = first[2:G + 2]
        return dict(num_groups=G, new_to_old=new_to_old, group_first=first, group_ranges=ranges,
                    out_offsets=off, out_ids=ids[:nnz])


    def _additional(self, fn, X, k, group_first, out_offsets, out_ids, cross_ids, *extra):
        X = np.ascontiguousarray(X, dtype=np.float32)
        n, d = X.shape
        G = group_first.shape[0] - 2
        gf = np.ascontiguousarray(group_first, dtype=np.uint32)
        oo = np.ascontiguousarray(out_offsets, dtype=np.uint64)
        oi = np.ascontiguousarray(out_ids, dtype=np.uint32)
        if oi.size == 0:
            oi = np.zeros(1, dtype=np.uint32)
        ci = np.ascontiguousarray(cross_ids, dtype=np.uint32).reshape(-1)
        count = fn(_p(X), n, d, k, G, _p(gf), _p(oo), _p(oi), _p(ci), *extra, 0, None, None)
        src = np.empty(max(count, 1), dtype=np.uint32)
        dst = np.empty(max(count, 1), dtype=np.uint32)
        fn(_p(X), n, d, k, G, _p(gf), _p(oo), _p(oi), _p(ci), *extra, count, _p(src), _p(dst))
        return src[:count], dst[:count]


class Oracle(_Lib):
    """The plain-C restatement."""

    def __init__(self, path: str = ORACLE_SO):
        super().__init__(path, "orc_")
        L = self.lib
        L.orc_l2.restype = c_float
        L.orc_l2.argtypes = [c_void_p, c_void_p, c_uint32, c_int]
        L.orc_cross_rows.restype = None
        L.orc_cross_rows.argtypes = [c_void_p, c_uint32, c_uint32, c_uint32, c_uint32, c_void_p, c_void_p,
                                     c_void_p, c_void_p, c_uint64, c_int, c_int, c_void_p, c_void_p]
        L.orc_cross_exact.restype = c_uint64
        L.orc_cross_exact.argtypes = [c_void_p, c_uint32, c_uint32, c_uint32, c_uint32, c_void_p, c_void_p,
                                      c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]
        L.orc_ung_search.restype = None
        L.orc_ung_search.argtypes = [c_void_p, c_uint32, c_uint32, c_void_p, c_void_p, c_void_p, c_uint32, c_void_p,
                                     c_void_p, c_uint32, c_uint32, c_int, c_int, c_void_p, c_void_p]
        L.orc_filtered_scan.restype = None
        L.orc_filtered_scan.argtypes = [c_void_p, c_uint32, c_void_p, c_void_p, c_uint32, c_void_p, c_void_p,
                                        c_uint32, c_int, c_int, c_void_p, c_void_p]
        L.orc_block_l2.restype = c_float
        L.orc_block_l2.argtypes = [c_void_p, c_void_p, c_uint32]
        L.orc_exact_knn_graph.restype = None
        L.orc_exact_knn_graph.argtypes = [c_void_p, c_uint32, c_uint32, c_void_p, c_uint32, c_uint32, c_uint32,
                                          c_uint32, c_uint32, c_uint32, c_uint32, c_int, c_void_p, c_void_p]
        L.orc_additional_edges.restype = c_uint64
        L.orc_additional_edges.argtypes = [c_void_p, c_uint32, c_uint32, c_uint32, c_uint32, c_void_p, c_void_p,
                                           c_void_p, c_void_p, c_int, c_uint64, c_void_p, c_void_p]

    def block_l2(self, a: np.ndarray, b: np.ndarray) -> float:
        """The distance of the reference's 128-thread kNN kernel (fast-math fp32)."""
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.float32)
        return self.lib.orc_block_l2(_p(a), _p(b), a.shape[0])

    def exact_knn_graph(self, X: np.ndarray, group_ranges: np.ndarray, candidate_k: int, final_degree: int,
                        head_keep: int, anchor_tail: int, anchor_slots: int, bidir_anchor: int, graph_stride: int,
                        num_threads: int = 0):
        """Rows [points x graph_stride] and entry points of the exact kNN seeding restatement."""
        X = np.ascontiguousarray(X, dtype=np.float32)
        r = np.ascontiguousarray(group_ranges, dtype=np.uint32)
        G = r.size // 2
        pts = int(np.sum(r[1::2].astype(np.int64) - r[0::2]))
        graph = np.zeros((max(pts, 1), graph_stride), dtype=np.uint32)
        entry = np.zeros(max(G, 1), dtype=np.uint32)
        self.lib.orc_exact_knn_graph(_p(X), X.shape[1], G, _p(r), candidate_k, final_degree, head_keep, anchor_tail,
                                     anchor_slots, bidir_anchor, graph_stride, num_threads, _p(graph), _p(entry))
        return graph[:pts], entry[:G]

    def additional_edges(self, X, k, group_first, out_offsets, out_ids, cross_ids, fused: int = L2_REFERENCE_BUILD):
        """(from, to) additional edges in the reference's materialised order."""
        return self._additional(self.lib.orc_additional_edges, X, k, group_first, out_offsets, out_ids, cross_ids,
                                fused)

    def ung_search(self, X, offsets, cols, Q, entry_offsets, entry_ids, L: int, K: int, num_threads: int = 0):
        """Greedy search of every query over the CSR graph: ids [nq x K] and distance counts [nq]."""
        X, off, c, Q, eo, ei = _search_args(X, offsets, cols, Q, entry_offsets, entry_ids)
        nq = Q.shape[0]
        ids = np.empty(max(nq * K, 1), dtype=np.uint32)
        cmps = np.empty(max(nq, 1), dtype=np.uint32)
        self.lib.orc_ung_search(_p(X), X.shape[0], X.shape[1], _p(off), _p(c), _p(Q), nq, _p(eo), _p(ei), L, K,
                                L2_REFERENCE_BUILD, num_threads, _p(ids), _p(cmps))
        return ids[:nq * K].reshape(nq, K), cmps[:nq]

    def filtered_scan(self, X, group_first, Q, target_offsets, target_ids, K: int, num_threads: int = 0):
        """Filtered brute-force ground truth: ids and distances [nq x K]."""
        X = np.ascontiguousarray(X, dtype=np.float32)
        Q = np.ascontiguousarray(Q, dtype=np.float32)
        gf = np.ascontiguousarray(group_first, dtype=np.uint32)
        to = np.ascontiguousarray(target_offsets, dtype=np.uint64)
        ti = np.ascontiguousarray(target_ids if len(target_ids) else [0], dtype=np.uint32)
        nq = Q.shape[0]
        ids = np.empty(max(nq * K, 1), dtype=np.uint32)
        dists = np.empty(max(nq * K, 1), dtype=np.float32)
        self.lib.orc_filtered_scan(_p(X), X.shape[1], _p(gf), _p(Q), nq, _p(to), _p(ti), K, L2_REFERENCE_BUILD,
                                   num_threads, _p(ids), _p(dists))
        return ids[:nq * K].reshape(nq, K), dists[:nq * K].reshape(nq, K)

    def l2(self, a: np.ndarray, b: np.ndarray, fused: int = L2_REFERENCE_BUILD) -> float:
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.float32)
        return self.lib.orc_l2(_p(a), _p(b), a.shape[0], fused)

    def cross_exact(self, X: np.ndarray, k: int, group_first: np.ndarray, out_offsets: np.ndarray,
                    out_ids: np.ndarray, source_mask: np.ndarray | None = None, num_threads: int = 0,
                    fused: int = L2_REFERENCE_BUILD):
        X = np.ascontiguousarray(X, dtype=np.float32)
        n, d = X.shape
        G = group_first.shape[0] - 2
        gf = np.ascontiguousarray(group_first, dtype=np.uint32)
        oo = np.ascontiguousarray(out_offsets, dtype=np.uint64)
        oi = np.ascontiguousarray(out_ids, dtype=np.uint32)
        if oi.size == 0:
            oi = np.zeros(1, dtype=np.uint32)
        sm = None if source_mask is None else np.ascontiguousarray(source_mask, dtype=np.uint8)
        ids = np.empty(n * k, dtype=np.uint32)
        dists = np.empty(n * k, dtype=np.float32)
        pairs = self.lib.orc_cross_exact(_p(X), n, d, k, G, _p(gf), _p(oo), _p(oi), _p(sm), num_threads, fused,
                                         _p(ids), _p(dists))
        return ids, dists, int(pairs)


    def cross_rows(self, X: np.ndarray, k: int, group_first: np.ndarray, out_offsets: np.ndarray,
                   out_ids: np.ndarray, rows: np.ndarray, num_threads: int = 0, fused: int = L2_REFERENCE_BUILD):
        """Exact top-k of the listed rows only; returns ids/dists of shape [len(rows), k]."""
        X = np.ascontiguousarray(X, dtype=np.float32)
        n, d = X.shape
        G = group_first.shape[0] - 2
        gf = np.ascontiguousarray(group_first, dtype=np.uint32)
        oo = np.ascontiguousarray(out_offsets, dtype=np.uint64)
        oi = np.ascontiguousarray(out_ids, dtype=np.uint32)
        if oi.size == 0:
            oi = np.zeros(1, dtype=np.uint32)
        rows = np.ascontiguousarray(rows, dtype=np.uint32)
        ids = np.empty((rows.size, k), dtype=np.uint32)
        dists = np.empty((rows.size, k), dtype=np.float32)
        self.lib.orc_cross_rows(_p(X), n, d, k, G, _p(gf), _p(oo), _p(oi), _p(rows), rows.size, num_threads,
                                fused, _p(ids), _p(dists))
        return ids, dists


class Reference(_Lib):
    """The reference's own compiled code behind ref_harness.cpp."""

    def __init__(self, path: str = REF_SO):
        super().__init__(path, "ungref_")
        L = self.lib
        L.ungref_label_graph_build.restype = c_void_p
        L.ungref_l2.restype = c_float
        L.ungref_l2.argtypes = [c_void_p, c_void_p, c_uint32]
        L.ungref_cross_exact.restype = c_uint64
        L.ungref_cross_exact.argtypes = [c_void_p, c_uint32, c_uint32, c_uint32, c_uint32, c_void_p, c_void_p,
                                         c_void_p, c_void_p, c_int, c_void_p, c_void_p]
        L.ungref_additional_edges.restype = c_uint64
        L.ungref_additional_edges.argtypes = [c_void_p, c_uint32, c_uint32, c_uint32, c_uint32, c_void_p,
                                              c_void_p, c_void_p, c_void_p, c_uint64, c_void_p, c_void_p]
        L.ungref_ung_search.restype = None
        L.ungref_ung_search.argtypes = [c_void_p, c_uint32, c_uint32, c_void_p, c_void_p, c_void_p, c_uint32,
                                        c_void_p, c_void_p, c_uint32, c_uint32, c_void_p]
        L.ungref_filtered_scan.restype = None
        L.ungref_filtered_scan.argtypes = [c_void_p, c_uint32, c_void_p, c_void_p, c_uint32, c_void_p, c_void_p,
                                           c_uint32, c_void_p, c_void_p]

    def ung_search(self, X, offsets, cols, Q, entry_offsets, entry_ids, L: int, K: int):
        """iterate_to_fixed_point over the reference's SearchQueue (single thread): ids [nq x K]."""
        X, off, c, Q, eo, ei = _search_args(X, offsets, cols, Q, entry_offsets, entry_ids)
        nq = Q.shape[0]
        ids = np.empty(max(nq * K, 1), dtype=np.uint32)
        self.lib.ungref_ung_search(_p(X), X.shape[0], X.shape[1], _p(off), _p(c), _p(Q), nq, _p(eo), _p(ei), L, K,
                                   _p(ids))
        return ids[:nq * K].reshape(nq, K)

    def filtered_scan(self, X, group_first, Q, target_offsets, target_ids, K: int):
        """FilteredScan::answer_one_query over the reference's SearchQueue: ids and distances [nq x K]."""
        X = np.ascontiguousarray(X, dtype=np.float32)
        Q = np.ascontiguousarray(Q, dtype=np.float32)
        gf = np.ascontiguousarray(group_first, dtype=np.uint32)
        to = np.ascontiguousarray(target_offsets, dtype=np.uint64)
        ti = np.ascontiguousarray(target_ids if len(target_ids) else [0], dtype=np.uint32)
        nq = Q.shape[0]
        ids = np.empty(max(nq * K, 1), dtype=np.uint32)
        dists = np.empty(max(nq * K, 1), dtype=np.float32)
        self.lib.ungref_filtered_scan(_p(X), X.shape[1], _p(gf), _p(Q), nq, _p(to), _p(ti), K, _p(ids), _p(dists))
        return ids[:nq * K].reshape(nq, K), dists[:nq * K].reshape(nq, K)

    def additional_edges(self, X, k, group_first, out_offsets, out_ids, cross_ids):
        """(from, to) additional edges in the reference's materialised order."""
        return self._additional(self.lib.ungref_additional_edges, X, k, group_first, out_offsets, out_ids, cross_ids)

    def graph_save_text(self, path: str, offsets: np.ndarray, cols: np.ndarray) -> None:
        """The CSR rows written by the reference's ANNS::Graph::save (graph.h:207-216)."""
        off = np.ascontiguousarray(offsets, dtype=np.uint64)
        c = np.ascontiguousarray(cols, dtype=np.uint32)
        if c.size == 0:
            c = np.zeros(1, dtype=np.uint32)
        self.lib.ungref_graph_save_text.argtypes = [ctypes.c_char_p, c_uint32, c_void_p, c_void_p]
        self.lib.ungref_graph_save_text(os.fsencode(path), off.size - 1, _p(off), _p(c))

    def l2(self, a: np.ndarray, b: np.ndarray) -> float:
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.float32)
        return self.lib.ungref_l2(_p(a), _p(b), a.shape[0])

    def cross_exact(self, X, k, group_first, out_offsets, out_ids, source_mask=None, num_threads: int = 0):
        X = np.ascontiguousarray(X, dtype=np.float32)
        n, d = X.shape
        G = group_first.shape[0] - 2
        gf = np.ascontiguousarray(group_first, dtype=np.uint32)
        oo = np.ascontiguousarray(out_offsets, dtype=np.uint64)
        oi = np.ascontiguousarray(out_ids, dtype=np.uint32)
        if oi.size == 0:
            oi = np.zeros(1, dtype=np.uint32)
        sm = None if source_mask is None else np.ascontiguousarray(source_mask, dtype=np.uint8)
        ids = np.empty(n * k, dtype=np.uint32)
        dists = np.empty(n * k, dtype=np.float32)
        pairs = self.lib.ungref_cross_exact(_p(X), n, d, k, G, _p(gf), _p(oo), _p(oi), _p(sm), num_threads,
                                            _p(ids), _p(dists))
        return ids, dists, int(pairs)


class ReferenceKnn:
    """The reference's own GPU exact kNN seeding: build_tagore_vamana_cuda_batch routed to
    build_fast_exact_cuda_batch / batched_exact_knn_graph_kernel
    (UNG/codes/src/tagore_graph_builder.cu:650-795, 1058-1340)."""

    def __init__(self, path: str = REF_KNN_SO):
        self.lib = ctypes.CDLL(path)
        self.lib.ungref_knn_batch.restype = c_int
        self.lib.ungref_knn_batch.argtypes = [c_void_p, c_uint32, c_uint32, c_void_p] + [c_uint32] * 7 + \
            [c_void_p, c_void_p]

    def exact_knn_graph(self, X: np.ndarray, group_ranges: np.ndarray, candidate_k: int, final_degree: int,
                        head_keep: int, anchor_tail: int, anchor_slots: int, bidir_anchor: int, graph_stride: int):
        """Rows [points x graph_stride] and entry points, groups = row ranges of X (their rows
        are passed to the reference concatenated in group order)."""
        r = np.ascontiguousarray(group_ranges, dtype=np.uint32)
        sizes = (r[1::2].astype(np.int64) - r[0::2]).astype(np.uint32)
        data = np.ascontiguousarray(np.concatenate([X[a:b] for a, b in zip(r[0::2], r[1::2])]), dtype=np.float32)
        pts = int(sizes.sum())
        graph = np.zeros((max(pts, 1), graph_stride), dtype=np.uint32)
        entry = np.zeros(max(sizes.size, 1), dtype=np.uint32)
        st = self.lib.ungref_knn_batch(_p(data), X.shape[1], sizes.size, _p(sizes), candidate_k, final_degree, head_keep,
                                       anchor_tail, anchor_slots, bidir_anchor, graph_stride, _p(graph), _p(entry))
        if st != 0:
            raise RuntimeError(f"reference kNN batch failed with status {st}")
        return graph[:pts], entry[:sizes.size]


def reference_knn() -> ReferenceKnn | None:
    return ReferenceKnn() if os.path.exists(REF_KNN_SO) else None


def oracle() -> Oracle:
    return Oracle()


def reference() -> Reference | None:
    return Reference() if os.path.exists(REF_SO) else None


def lng_sets(out_offsets: np.ndarray, out_ids: np.ndarray, num_groups: int) -> list[frozenset]:
    return [frozenset(out_ids[out_offsets[g]:out_offsets[g + 1]].tolist()) for g in range(num_groups + 1)]


def _search_args(X, offsets, cols, Q, entry_offsets, entry_ids):
    X = np.ascontiguousarray(X, dtype=np.float32)
    off = np.ascontiguousarray(offsets, dtype=np.uint64)
    c = np.ascontiguousarray(cols if len(cols) else [0], dtype=np.uint32)
    Q = np.ascontiguousarray(Q, dtype=np.float32)
    eo = np.ascontiguousarray(entry_offsets, dtype=np.uint64)
    ei = np.ascontiguousarray(entry_ids if len(entry_ids) else [0], dtype=np.uint32)
    return X, off, c, Q, eo, ei


def query_groups(set_offsets: np.ndarray, set_labels: np.ndarray, query_offsets: np.ndarray,
                 query_labels: np.ndarray):
    """Per query label set, over the base groups 1..G and their sorted label sets:

    * the containment targets, every group whose set includes the query's (ascending
      group id): the groups FilteredScan scans (filtered_scan.cpp:131-154);
    * the minimal ones among them, no other target's set strictly inside theirs: the
      entry groups of a containment query (get_min_super_sets with avoid_self false,
      UNG/codes/src/uni_nav_graph_label_graph.cpp:45-54; get_entry_points,
      UNG/codes/src/uni_nav_graph_search_backend.cpp:169-198).

    Returned as two CSR pairs (offsets uint64 [nq+1], group ids uint32)."""
    G = set_offsets.shape[0] - 2
    so = set_offsets.astype(np.int64)
    qo = query_offsets.astype(np.int64)
    labels = np.unique(np.concatenate([set_labels, query_labels]).astype(np.int64))
    if labels.size > 63:
        raise ValueError("query_groups handles at most 63 distinct labels")
    pos = np.searchsorted(labels, set_labels.astype(np.int64))
    owner = np.repeat(np.arange(G + 1), np.diff(so))
    masks = np.zeros(G + 1, dtype=np.int64)
    np.bitwise_or.at(masks, owner, np.left_shift(np.int64(1), pos))
    qpos = np.searchsorted(labels, query_labels.astype(np.int64))
    nq = qo.shape[0] - 1
    t_off, t_ids, m_off, m_ids = [0], [], [0], []
    exact = {int(m): g for g, m in enumerate(masks.tolist()) if g > 0}
    for q in range(nq):
        qm = 0
        for p in qpos[qo[q]:qo[q + 1]].tolist():
            qm |= 1 << p
        tg = np.nonzero((masks[1:] & qm) == qm)[0] + 1
        if qm in exact:                     # the query's own set is a group: the only minimal one
            mins = np.array([exact[qm]])
        else:
            tm = masks[tg]
            inner = ((tm[None, :] & tm[:, None]) == tm[None, :]) & (tm[None, :] != tm[:, None])
            mins = tg[~inner.any(axis=1)]
        t_ids.append(tg)
        m_ids.append(mins)
        t_off.append(t_off[-1] + tg.size)
        m_off.append(m_off[-1] + mins.size)
    cat = lambda parts: np.concatenate(parts).astype(np.uint32) if parts else np.zeros(0, np.uint32)
    return np.array(t_off, dtype=np.uint64), cat(t_ids), np.array(m_off, dtype=np.uint64), cat(m_ids)


def entry_points(group_first: np.ndarray, group_entry: np.ndarray, entry_offsets: np.ndarray,
                 entry_groups: np.ndarray, num_entry_points: int = 16, seed: int = 0):
    """Entry vectors of every query, get_entry_points_given_group_id
    (UNG/codes/src/uni_nav_graph_search_backend.cpp:200-228) per entry group in order:
    a group of at most num_entry_points vectors gives all of them; a larger one gives its
    entry point, then for i = 1 .. num_entry_points-1 the vector first + i whenever the
    random draw of that step hits a vector not drawn before (the reference appends
    first + i, not the drawn vector).  The reference draws with the C library's rand(),
    shared by its search threads; here each query has its own seeded generator.
    group_entry holds each group's entry point as a local index (0 .. size-1)."""
    nq = entry_offsets.shape[0] - 1
    off, ids = [0], []
    for q in range(nq):
        rng = np.random.default_rng([seed, q])
        marked = set()
        for g in entry_groups[entry_offsets[q]:entry_offsets[q + 1]].tolist():
            first, last = int(group_first[g]), int(group_first[g + 1])
            size = last - first
            if size <= num_entry_points:
                ids += range(first, last)
                continue
            ep = first + int(group_entry[g])
            marked.add(ep)
            ids.append(ep)
            draws = rng.integers(0, size, size=num_entry_points - 1)
            for i in range(1, num_entry_points):
                r = first + int(draws[i - 1])
                if r not in marked:
                    marked.add(r)
                    ids.append(first + i)
        off.append(len(ids))
    return np.array(off, dtype=np.uint64), np.array(ids, dtype=np.uint32)


def recall_at_k(result_ids: np.ndarray, truth_ids: np.ndarray) -> float:
    """Mean over queries of |result ∩ truth| / |truth| (truth without empty slots)."""
    tot, hit = 0, 0
    for r, t in zip(result_ids, truth_ids):
        ts = set(t.tolist()) - {0xFFFFFFFF}
        tot += len(ts)
        hit += len(ts & set(r.tolist()))
    return hit / max(tot, 1)
