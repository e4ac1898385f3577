"""Inputs that stress the tensor-core route's rounding certificate.

Each case is a reordered base matrix with hand-made groups (group g owns rows
[first[g], first[g+1])) and out-neighbour lists, so the certificate meets:

* ``norm_span``   source and target rows whose norms span 1e-3 .. 1e3 (log-uniform) in
                  one group pair: the bound, scaled by the largest target norm, is far
                  above the distances of the small rows;
* ``subnormal``   one huge element fixes the power-of-two scale, so that every other
                  element of the fp16 operand falls below fp16's normal range;
* ``near_normal`` data scaled so the operand's elements straddle the smallest normal
                  fp16 value (2^-14);
* ``exact_only``  one element above the fp16 operand's range for any scale: every row
                  must go to the exact rescan (its distances overflow to +inf);
* ``offset``      1000 + U[0, 1): the centring before rounding carries the precision;
* ``ties``        a coarse grid of values with many equal distances and duplicates.

The expected rows come from the CPU oracle (or the reference's own compiled scan),
never from the device.
"""
import numpy as np

CASES = ["norm_span", "subnormal", "near_normal", "exact_only", "offset", "ties"]


def _groups(sizes, outs):
    """first [G+2] and out CSR for groups 1..G of the given sizes (out lists 1-based)."""
    G = len(sizes)
    first = np.zeros(G + 2, dtype=np.uint32)
    first[2:] = np.cumsum(sizes)
    first[1] = 0
    off = np.zeros(G + 2, dtype=np.uint64)
    ids = []
    for g in range(1, G + 1):
        off[g] = len(ids)
        ids += outs.get(g, [])
    off[G + 1] = len(ids)
    ranges = np.zeros(2 * (G + 1), dtype=np.uint32)
    ranges[2::2] = first[1:G + 1]
    ranges[3::2] = first[2:G + 2]
    return first, ranges, off, np.array(ids if ids else [0], dtype=np.uint32)[:len(ids)]


def make_case(name: str, seed: int = 0):
    """(X [n x d] fp32 in reordered order, k, group_first, group_ranges, out_offsets, out_ids)."""
    rng = np.random.default_rng([seed, CASES.index(name)])
    # five groups: 1 -> {2, 3}, 4 -> {2, 5}, 2 -> {5}; 3 and 5 have no targets
    sizes = [700, 1500, 600, 300, 900]
    outs = {1: [2, 3], 4: [2, 5], 2: [5]}
    d, k = 128, 6
    n = sum(sizes)
    if name == "norm_span":
        X = rng.standard_normal((n, d)).astype(np.float32)
        X /= np.linalg.norm(X, axis=1, keepdims=True)
        X *= (10.0 ** rng.uniform(-3, 3, size=(n, 1))).astype(np.float32)
    elif name == "subnormal":
        X = (rng.standard_normal((n, d)) * 1e-6).astype(np.float32)
        X[5, 0] = 3.0e3       # sets the scale: s = 8, so s * 1e-6 is below 2^-14
    elif name == "near_normal":
        X = (rng.standard_normal((n, d)) * 2e-3).astype(np.float32)
        X[:, 1::2] *= np.float32(2e-3)  # half of the columns at ~4e-6
        X[7, 3] = 1.0         # the scale: s = 2^14, so those columns land at ~6.5e-5, around 2^-14
    elif name == "exact_only":
        X = rng.standard_normal((n, d)).astype(np.float32)
        X[11, 5] = np.float32(1e24)  # beyond 2^75: no power-of-two scale fits fp16
        d = 64
        X = np.ascontiguousarray(X[:, :d])
    elif name == "offset":
        X = (1000.0 + rng.random((n, d))).astype(np.float32)
    elif name == "ties":
        d, k = 13, 8
        X = rng.integers(0, 3, size=(n, d)).astype(np.float32)
        X[100:140] = X[60:100]   # exact duplicates inside group 1
    else:
        raise ValueError(name)
    first, ranges, off, ids = _groups(sizes, outs)
    return np.ascontiguousarray(X, dtype=np.float32), k, first, ranges, off, ids
