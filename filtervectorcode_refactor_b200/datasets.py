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

Large inputs are drawn in blocks of 2^16 rows on several threads, block b from its
own stream: vectors ``default_rng([seed, 1, b])`` when n * d >= 2^28 (configurations
3 and 4), labels ``default_rng([seed, 0, b])`` (all u of the block, then its Gumbel
noise) when n > 2^21 (configuration 4).  Smaller inputs keep the single streams
above, so the fixtures made from them stay valid.
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

BLOCK_ROWS = 1 << 16
PARALLEL_VECTOR_ELEMS = 1 << 28
PARALLEL_LABEL_ROWS = 1 << 21


def _threads(threads: int = 0) -> int:
    return threads if threads > 0 else min(32, os.cpu_count() or 1)


def reorder_rows(X: np.ndarray, new_to_old: np.ndarray, threads: int = 0) -> np.ndarray:
    """X[new_to_old] (rows gathered into a new contiguous array) on several threads."""
    idx = np.ascontiguousarray(new_to_old).astype(np.intp, copy=False)
    out = np.empty((idx.shape[0],) + X.shape[1:], dtype=X.dtype)
    step = 1 << 18

    def part(a: int) -> None:
        b = min(idx.shape[0], a + step)
        np.take(X, idx[a:b], axis=0, out=out[a:b])

    with ThreadPoolExecutor(_threads(threads)) as ex:
        list(ex.map(part, range(0, idx.shape[0], step)))
    return out

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
    logw = -zipf * np.log(np.arange(1, vocab + 1, dtype=np.float64))
    if n > PARALLEL_LABEL_ROWS:
        return _make_labels_blocked(n, vocab, umin, umax, logw, seed)
    rng = np.random.default_rng(seed)
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


def _make_labels_blocked(n: int, vocab: int, umin: int, umax: int, logw: np.ndarray, seed: int,
                         threads: int = 0) -> tuple[np.ndarray, np.ndarray]:
    blocks = range((n + BLOCK_ROWS - 1) // BLOCK_ROWS)
    rngs = [np.random.default_rng([seed, 0, b]) for b in blocks]
    u = np.empty(n, dtype=np.int64)

    def draw_u(b: int) -> None:
        a = b * BLOCK_ROWS
        u[a:min(n, a + BLOCK_ROWS)] = rngs[b].integers(umin, umax + 1, size=min(n, a + BLOCK_ROWS) - a)

    with ThreadPoolExecutor(_threads(threads)) as ex:
        list(ex.map(draw_u, blocks))
    offsets = np.zeros(n + 1, dtype=np.uint64)
    np.cumsum(u.astype(np.uint64), out=offsets[1:])
    labels = np.empty(int(offsets[-1]), dtype=np.uint32)

    def fill(b: int) -> None:
        a = b * BLOCK_ROWS
        e = min(n, a + BLOCK_ROWS)
        g = rngs[b].gumbel(size=(e - a, vocab)) + logw[None, :]
        # every column vocab - u (u in umin..umax) in its sorted place: row i's u_i-th largest
        thr = np.partition(g, list(range(vocab - umax, vocab - umin + 1)), axis=1)
        cut = thr[np.arange(e - a), vocab - u[a:e]]
        _, cols = np.nonzero(g >= cut[:, None])
        labels[int(offsets[a]):int(offsets[e])] = cols.astype(np.uint32) + 1

    with ThreadPoolExecutor(_threads(threads)) as ex:
        list(ex.map(fill, blocks))
    return offsets, labels


def make_vectors(n: int, d: int, dist: str, normalize: bool, seed: int, threads: int = 0) -> np.ndarray:
    if dist not in ("normal", "uniform"):
        raise ValueError(dist)
    if n * d >= PARALLEL_VECTOR_ELEMS:
        X = np.empty((n, d), dtype=np.float32)

        def fill(b: int) -> None:
            a = b * BLOCK_ROWS
            e = min(n, a + BLOCK_ROWS)
            rng = np.random.default_rng([seed, 1, b])
            if dist == "normal":
                rng.standard_normal((e - a, d), dtype=np.float32, out=X[a:e])
            else:
                rng.random((e - a, d), dtype=np.float32, out=X[a:e])
            if normalize:
                nrm = np.sqrt(np.einsum("ij,ij->i", X[a:e], X[a:e], dtype=np.float32))
                nrm[nrm == 0] = 1
                X[a:e] /= nrm[:, None]

        with ThreadPoolExecutor(_threads(threads)) as ex:
            list(ex.map(fill, range((n + BLOCK_ROWS - 1) // BLOCK_ROWS)))
        return X
    rng = np.random.default_rng([seed, 1])
    if dist == "normal":
        X = rng.standard_normal((n, d), dtype=np.float32)
    else:
        X = rng.random((n, d), dtype=np.float32)
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
