"""Seeded synthetic inputs with the shapes of the benchmark configurations.

The reference measured on Amazon / CelebA / SIFT-derived datasets that are not
available here; these generators stand in for them with the distributions the
benchmark configurations name.  Both the oracle and the GPU path read the same
arrays, so parity does not depend on the generator.

Label sets: u ~ Uniform{umin..umax} distinct labels per vector, drawn without
replacement from Zipf(s) weights proportional to 1/r^s over labels 1..V by the
Gumbel-top-u trick (add Gumbel noise to log-weights, keep the u largest), then
sorted.  Stream: ``numpy.random.default_rng(seed)`` draws all u first, then the
Gumbel noise row by row.  Vectors: ``numpy.random.default_rng([seed, 1])``.
"""
from __future__ import annotations

import numpy as np

CONFIGS = {
    1: dict(name="cfg1_100k_d128_v10", n=100_000, d=128, vocab=10, umin=1, umax=3, zipf=1.2,
            dist="normal", normalize=False, k=6),
    2: dict(name="cfg2_1M_d128_v30_l2norm", n=1_000_000, d=128, vocab=30, umin=1, umax=4, zipf=1.0,
            dist="normal", normalize=True, k=6),
    3: dict(name="cfg3_1M_d960_v12_uniform", n=1_000_000, d=960, vocab=12, umin=1, umax=3, zipf=1.5,
            dist="uniform", normalize=False, k=16),
    4: dict(name="cfg4_10M_d96_v40", n=10_000_000, d=96, vocab=40, umin=1, umax=5, zipf=1.0,
            dist="normal", normalize=False, k=6),
}

# Configuration 5: the configuration-2 index searched by nq queries, each with a
# label set of 1-2 labels from the same Zipf(1.0) over 30 (containment filter);
# greedy search L = 100, top-10.
QUERIES = dict(nq=10_240, d=128, vocab=30, umin=1, umax=2, zipf=1.0, dist="normal", normalize=False,
               L=100, K=10, num_entry_points=16)


def make_labels(n: int, vocab: int, umin: int, umax: int, zipf: float, seed: int,
                chunk: int = 1 << 19) -> tuple[np.ndarray, np.ndarray]:
    """Label sets as CSR (offsets uint64 [n+1], labels uint32, each row ascending)."""
    rng = np.random.default_rng(seed)
    logw = -zipf * np.log(np.arange(1, vocab + 1, dtype=np.float64))
    u = rng.integers(umin, umax + 1, size=n)
    counts = u.astype(np.uint64)
    offsets = np.zeros(n + 1, dtype=np.uint64)
    np.cumsum(counts, out=offsets[1:])
    labels = np.empty(int(offsets[-1]), dtype=np.uint32)
    for a in range(0, n, chunk):
        b = min(n, a + chunk)
        g = rng.gumbel(size=(b - a, vocab)) + logw[None, :]
        srt = np.sort(g, axis=1)
        thr = srt[np.arange(b - a), vocab - u[a:b]]
        mask = g >= thr[:, None]
        _, cols = np.nonzero(mask)
        labels[int(offsets[a]):int(offsets[b])] = cols.astype(np.uint32) + 1
    return offsets, labels


def make_vectors(n: int, d: int, dist: str, normalize: bool, seed: int) -> np.ndarray:
    rng = np.random.default_rng([seed, 1])
    if dist == "normal":
        X = rng.standard_normal((n, d), dtype=np.float32)
    elif dist == "uniform":
        X = rng.random((n, d), dtype=np.float32)
    else:
        raise ValueError(dist)
    if normalize:
        nrm = np.sqrt(np.einsum("ij,ij->i", X, X, dtype=np.float32))
        nrm[nrm == 0] = 1
        X /= nrm[:, None]
    return X


def make_config(cfg: int, seed: int = 0, n: int | None = None) -> dict:
    """Inputs of configuration ``cfg`` (optionally with fewer points, same distributions)."""
    c = dict(CONFIGS[cfg])
    if n is not None:
        c["n"] = n
    off, lab = make_labels(c["n"], c["vocab"], c["umin"], c["umax"], c["zipf"], seed)
    X = make_vectors(c["n"], c["d"], c["dist"], c["normalize"], seed)
    c.update(label_offsets=off, labels=lab, X=X, seed=seed)
    return c


def make_queries(seed: int = 0, nq: int | None = None) -> dict:
    """Configuration-5 queries: vectors from ``default_rng([seed, 2])``, label sets from
    the label stream seeded ``seed + 1_000_003``."""
    c = dict(QUERIES)
    if nq is not None:
        c["nq"] = nq
    off, lab = make_labels(c["nq"], c["vocab"], c["umin"], c["umax"], c["zipf"], seed + 1_000_003)
    rng = np.random.default_rng([seed, 2])
    Q = rng.standard_normal((c["nq"], c["d"]), dtype=np.float32)
    c.update(label_offsets=off, labels=lab, Q=Q, seed=seed)
    return c
