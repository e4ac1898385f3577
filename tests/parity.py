"""Row comparison used by every parity test.

The contract (north star): neighbour ids identical except at fp32 distance ties
with |dd|/d <= 1e-5, per-vector edge recall >= 0.999.  This build reproduces the
reference's fp32 summation order, so the tests demand more: ids equal and distance
bits equal, row by row.  On failure the message also reports whether the rows would
pass the tie-tolerant contract.
"""
import numpy as np

TIE_RTOL = 1e-5


def tie_tolerant_equal(ids_a, d_a, ids_b, d_b) -> bool:
    if np.array_equal(ids_a, ids_b):
        return True
    ok = (ids_a == 0xFFFFFFFF) == (ids_b == 0xFFFFFFFF)
    fin = np.isfinite(d_a) & np.isfinite(d_b)
    close = np.abs(d_a[fin] - d_b[fin]) <= TIE_RTOL * np.maximum(np.abs(d_b[fin]), 1e-30)
    return bool(ok.all() and close.all())


def assert_rows_match(ids, dists, ref_ids, ref_dists, k, rows=None):
    ids = ids.reshape(-1, k)
    ref_ids = ref_ids.reshape(-1, k)
    dists = dists.reshape(-1, k)
    ref_dists = ref_dists.reshape(-1, k)
    if rows is not None:
        ids, dists = ids[rows], dists[rows]
        ref_ids, ref_dists = ref_ids[rows], ref_dists[rows]
    bad = np.nonzero(~(np.all(ids == ref_ids, axis=1) &
                       np.all(dists.view(np.uint32) == ref_dists.view(np.uint32), axis=1)))[0]
    if bad.size:
        tol = sum(tie_tolerant_equal(ids[i], dists[i], ref_ids[i], ref_dists[i]) for i in bad)
        recall = np.mean([len(set(ids[i]) & set(ref_ids[i])) / max(1, len(set(ref_ids[i]) - {0xFFFFFFFF}))
                          for i in bad])
        i = bad[0]
        raise AssertionError(
            f"{bad.size} of {ids.shape[0]} rows differ ({tol} within the tie tolerance, mean recall of the "
            f"differing rows {recall:.4f}); first row {i if rows is None else rows[i]}: "
            f"got {ids[i].tolist()} {dists[i].tolist()} expected {ref_ids[i].tolist()} {ref_dists[i].tolist()}")


def row_groups(group_ranges, n):
    """Group id (1..G) of every row; 0 for rows outside every group."""
    gr = group_ranges.reshape(-1, 2).astype(np.int64)
    sizes = gr[1:, 1] - gr[1:, 0]
    rg = np.zeros(n, dtype=np.int64)
    rows = np.repeat(np.arange(1, gr.shape[0]), sizes)
    starts = np.repeat(gr[1:, 0], sizes)
    rg[starts + (np.arange(rows.size) - np.repeat(np.cumsum(sizes) - sizes, sizes))] = rows
    return rg


def check_row_properties_fast(ids, dists, k, group_ranges, out_offsets, out_ids, rows):
    """check_row_properties over many rows at once (vectorised); returns the number of
    rows checked."""
    gr = group_ranges.reshape(-1, 2).astype(np.int64)
    G = gr.shape[0] - 1
    sizes = gr[:, 1] - gr[:, 0]
    oo = out_offsets.astype(np.int64)
    oi = out_ids.astype(np.int64)
    n = ids.size // k
    rg = row_groups(group_ranges, n)
    src = np.repeat(np.arange(G + 1), np.diff(oo[:G + 2]))
    union = np.zeros(G + 1, dtype=np.int64)
    np.add.at(union, src, sizes[oi])
    edge_keys = np.unique(src * (G + 1) + oi)
    rows = np.asarray(rows, dtype=np.int64)
    I = ids.reshape(-1, k)[rows].astype(np.int64)
    D = dists.reshape(-1, k)[rows]
    f = rg[rows]
    want = np.minimum(k, union[f])
    valid = I != 0xFFFFFFFF
    expect = np.arange(k)[None, :] < want[:, None]
    bad = np.nonzero(np.any(valid != expect, axis=1))[0]
    assert bad.size == 0, f"row {rows[bad[0]]}: ids {I[bad[0]].tolist()} want {want[bad[0]]} edges"
    assert np.all(np.isfinite(D[valid])) and np.all(np.isinf(D[~valid]))
    pair = valid[:, 1:] & valid[:, :-1]
    order = (D[:, 1:] > D[:, :-1]) | ((D[:, 1:] == D[:, :-1]) & (I[:, 1:] > I[:, :-1]))
    bad = np.nonzero(np.any(pair & ~order, axis=1))[0]
    assert bad.size == 0, f"row {rows[bad[0]]} not sorted: {I[bad[0]].tolist()} {D[bad[0]].tolist()}"
    tg = np.where(valid, rg[np.where(valid, I, 0)], 0)
    keys = f[:, None] * (G + 1) + tg
    member = np.isin(keys, edge_keys) | ~valid
    bad = np.nonzero(~np.all(member, axis=1))[0]
    assert bad.size == 0, f"row {rows[bad[0]]}: an id outside the union of its out-groups {I[bad[0]].tolist()}"
    return rows.size


def check_row_properties(ids, dists, k, group_ranges, out_offsets, out_ids, rows):
    """Size-independent properties of any output row: sorted by (distance, id),
    ids drawn from the union of the row's LNG out-groups, sentinels only at the end,
    and as many edges as min(k, union size)."""
    G = group_ranges.shape[0] // 2 - 1
    gr = group_ranges.reshape(-1, 2).astype(np.int64)
    row_group = np.zeros(int(gr[1:, 1].max()) if G else 0, dtype=np.int64)
    for g in range(1, G + 1):
        row_group[gr[g, 0]:gr[g, 1]] = g
    ids = ids.reshape(-1, k)
    dists = dists.reshape(-1, k)
    for r in rows:
        f = row_group[r]
        outs = out_ids[out_offsets[f]:out_offsets[f + 1]].astype(np.int64)
        union = int(sum(gr[t, 1] - gr[t, 0] for t in outs))
        want = min(k, union)
        row_ids, row_d = ids[r], dists[r]
        valid = row_ids != 0xFFFFFFFF
        assert valid.sum() == want, (r, row_ids, want)
        assert np.all(valid[:want]) and not np.any(valid[want:])
        v_ids = row_ids[:want].astype(np.int64)
        v_d = row_d[:want]
        assert np.all(np.isfinite(v_d)) and np.all(np.isinf(row_d[want:]))
        order_ok = (v_d[1:] > v_d[:-1]) | ((v_d[1:] == v_d[:-1]) & (v_ids[1:] > v_ids[:-1]))
        assert np.all(order_ok), (r, v_ids, v_d)
        assert set(row_group[v_ids].tolist()) <= set(outs.tolist()), (r, v_ids, outs)
