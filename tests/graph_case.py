"""The merged per-point adjacency of build_cross_group_edges, assembled on the host from
the golden fixtures (the reference harness's cross and additional edges)."""
import numpy as np


def expected_merged_graph(g, intra_off, intra_local, with_additional=True):
    """The reference's build_cross_group_edges result per point, assembled on the host
    from the golden outputs: intra edges + the group's first row (add_offset), cross
    edges nearest first, additional edges in the materialised list's order."""
    n = g["Xr"].shape[0]
    k = g["k"]
    first = g["group_first"].astype(np.int64)
    grp = np.searchsorted(first[1:], np.arange(n), side="right")  # group id of each row
    ids = g["ids"].reshape(n, k)
    add = {}
    if with_additional:
        for f, t in zip(g["add_from"].tolist(), g["add_to"].tolist()):
            add.setdefault(f, []).append(t)
    rows = []
    for v in range(n):
        row = [int(x) + int(first[grp[v]]) for x in intra_local[intra_off[v]:intra_off[v + 1]]]
        row += [int(x) for x in ids[v] if x != 0xFFFFFFFF]
        row += add.get(v, [])
        rows.append(row)
    off = np.zeros(n + 1, dtype=np.uint64)
    off[1:] = np.cumsum([len(r) for r in rows])
    return off, np.array([x for r in rows for x in r], dtype=np.uint32)


def local_intra_graph(g, seed):
    """A random intra-group graph with group-local ids (each point: up to 5 members of its group)."""
    n = g["Xr"].shape[0]
    first = g["group_first"].astype(np.int64)
    grp = np.searchsorted(first[1:], np.arange(n), side="right")
    size = first[grp + 1] - first[grp]
    rng = np.random.default_rng(seed)
    deg = np.minimum(rng.integers(0, 6, size=n), size)
    off = np.zeros(n + 1, dtype=np.uint64)
    off[1:] = np.cumsum(deg)
    cols = (rng.random(int(off[-1])) * np.repeat(size, deg)).astype(np.uint32)
    return off, cols
