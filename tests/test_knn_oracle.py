"""The exact kNN seeding restatement (oracle side, CPU).

The reference's seeding kernel runs only on a GPU: the GPU tests pin this restatement
and the device path to it (tests/test_knn_gpu.py, oracle/_ref/libungref_knn.so).  What
is checked here, on the CPU: the distance order of its 128-thread block, restated
independently with numpy (for d <= 128 every per-thread partial is one rounded square,
and fp32 numpy arithmetic rounds like the device), and the row layout rules on small
hand-checked cases."""
import numpy as np
import pytest

import oracle as O


def block_l2_numpy(a: np.ndarray, b: np.ndarray) -> np.float32:
    d = a.shape[0]
    part = np.zeros(128, dtype=np.float32)
    diff = (a - b).astype(np.float32)
    part[:d] = diff * diff
    def warp(p):
        v = p.copy()
        off = 16
        while off:
            v[:off] = v[:off] + v[off:2 * off]
            off //= 2
        return v[0]
    w = [warp(part[32 * j:32 * j + 32]) for j in range(4)]
    return np.float32(np.float32(w[0] + w[2]) + np.float32(w[1] + w[3]))


@pytest.mark.parametrize("d", [1, 7, 13, 32, 33, 96, 100, 128])
def test_block_l2_matches_independent_restatement(d):
    rng = np.random.default_rng(d)
    orc = O.oracle()
    for _ in range(50):
        a = rng.standard_normal(d).astype(np.float32)
        b = rng.standard_normal(d).astype(np.float32)
        assert np.float32(orc.block_l2(a, b)).view(np.uint32) == block_l2_numpy(a, b).view(np.uint32)


def test_layout_head_and_anchors():
    # 40 points on a line: nearest neighbours are the adjacent indices
    X = np.arange(40, dtype=np.float32)[:, None] * np.ones((1, 4), dtype=np.float32)
    graph, entry = O.oracle().exact_knn_graph(X, np.array([0, 40], dtype=np.uint32), 64, 32, 24, 1, 0, 0, 33)
    assert entry.tolist() == [0]
    row = graph[10]
    assert row[0] == 32
    near = row[1:25].tolist()
    # the 24 nearest of point 10, (distance, id) order: 9, 11, 8, 12, ...
    exp = sorted([x for x in range(40) if x != 10], key=lambda x: (abs(x - 10), x))[:24]
    assert near == exp
    # anchors: hops (t+1)*n/9 from 10, skipping duplicates by walking forward
    anchors = row[25:33].tolist()
    assert len(set(near + anchors)) == 32 and 10 not in anchors


def test_small_groups_pad_with_self():
    X = np.random.default_rng(3).standard_normal((3, 5)).astype(np.float32)
    graph, _ = O.oracle().exact_knn_graph(X, np.array([0, 1, 1, 3], dtype=np.uint32), 64, 32, 24, 1, 0, 0, 33)
    assert graph[0, 0] == 0 and np.all(graph[0, 1:] == 0)          # singleton: no edges, padded with itself
    assert graph[1, 0] == 1 and graph[1, 1] == 1 and np.all(graph[1, 2:] == 0)
    assert graph[2, 0] == 1 and graph[2, 1] == 0 and np.all(graph[2, 2:] == 1)
