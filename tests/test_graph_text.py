"""The graph in the reference's on-disk text format (ungx_graph_save_text) against the
reference's own ANNS::Graph::save (UNG/codes/include/graph.h:207-216, linked from the
reference sources into oracle/_ref) and a plain restatement of that format: rows
longer than NeighborList's 64 inline slots, empty rows, the largest ids."""
import numpy as np
import pytest

import oracle as O
from filtervectorcode_refactor_b200 import _native as nat


def restate(offsets, cols):
    lines = []
    for v in range(offsets.size - 1):
        row = cols[offsets[v]:offsets[v + 1]]
        lines.append(f"{v} " + "".join(f"{int(c)} " for c in row) + "\n")
    return "".join(lines).encode()


def csr(seed, n):
    rng = np.random.default_rng(seed)
    deg = rng.integers(0, 90, n)
    deg[::7] = 0
    deg[min(3, n - 1)] = 200                       # beyond the 64 inline slots
    off = np.zeros(n + 1, dtype=np.uint64)
    off[1:] = np.cumsum(deg)
    cols = rng.integers(0, 2**32 - 1, int(off[-1]), dtype=np.uint64).astype(np.uint32)
    cols[:5] = [0, 9, 10, 2**32 - 2, 4294967295 - 1]
    return off, cols


@pytest.mark.parametrize("n", [1, 70000, 140001])
def test_graph_text_matches_reference(tmp_path, n):
    off, cols = csr(n, n)
    ours = tmp_path / "ours"
    nat.graph_save_text(str(ours), off, cols)
    data = ours.read_bytes()
    assert data == restate(off, cols)
    ref = O.reference()
    if ref is None:
        pytest.skip("the reference harness (oracle/_ref) is not built")
    theirs = tmp_path / "theirs"
    ref.graph_save_text(str(theirs), off, cols)
    assert data == theirs.read_bytes()


def test_graph_text_empty_and_errors(tmp_path):
    path = tmp_path / "g"
    nat.graph_save_text(str(path), np.zeros(1, dtype=np.uint64), np.zeros(0, dtype=np.uint32))
    assert path.read_bytes() == b""
    with pytest.raises(nat.UngxError):
        nat.graph_save_text(str(path), np.array([0, 3, 2], dtype=np.uint64), np.zeros(3, dtype=np.uint32))
    with pytest.raises(nat.UngxError):
        nat.graph_save_text(str(tmp_path / "missing" / "g"), np.array([0, 1], dtype=np.uint64),
                            np.zeros(1, dtype=np.uint32))
