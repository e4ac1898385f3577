"""The C ABI library: loads on a machine without a GPU, exports every symbol the
public headers declare, and its host-only logic (planning, sharding, CSR) holds."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT, have_gpu
from filtervectorcode_refactor_b200 import _native as nat


def declared_functions():
    names = []
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not h.endswith(".h"):
            continue
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\**\s*(ungx_[a-z_0-9]+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 20
    lib = ctypes.CDLL(nat.LIB_PATH)
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(nat.EXPORTED) | (set(names) - set(nat.EXPORTED))
    for n in nat.EXPORTED:
        assert n in names, f"binding for undeclared symbol {n}"


def test_status_strings():
    assert nat.lib.ungx_status_string(0) == b"ok"
    assert nat.lib.ungx_status_string(nat.UNGX_ERR_TIMEOUT) == b"timeout"


@pytest.mark.skipif(have_gpu(), reason="checks the no-device error path")
def test_context_create_without_device_fails_cleanly():
    with pytest.raises(nat.UngxError) as e:
        nat.Context(0)
    assert e.value.status == nat.UNGX_ERR_NO_DEVICE


def _toy_problem(**kw):
    # groups: 1 = rows [0,5), 2 = [5,9), 3 = [9,9) empty, 4 = [9,12); edges 1->2, 1->3, 2->4
    ranges = np.array([0, 0, 0, 5, 5, 9, 9, 9, 9, 12], dtype=np.uint32)
    off = np.array([0, 0, 2, 3, 3, 3], dtype=np.uint64)
    ids = np.array([2, 3, 4], dtype=np.uint32)
    return nat.Problem(12, 4, 3, ranges, off, ids, **kw)


def test_shard_rows_partition():
    full = _toy_problem().shard_rows()
    assert full.tolist() == list(range(12))
    for S in (2, 3, 5):
        parts = [_toy_problem(shard_rank=r, shard_count=S).shard_rows() for r in range(S)]
        allr = np.sort(np.concatenate(parts))
        assert allr.tolist() == list(range(12))


@pytest.mark.parametrize("bad", ["range", "edge", "shard"])
def test_plan_validation(bad):
    ranges = np.array([0, 0, 0, 5, 5, 9], dtype=np.uint32)
    off = np.array([0, 0, 1, 1], dtype=np.uint64)
    ids = np.array([2], dtype=np.uint32)
    kw = {}
    if bad == "range":
        ranges[3] = 50
    elif bad == "edge":
        ids[0] = 7
    else:
        kw = dict(shard_rank=2, shard_count=2)
    p = nat.Problem(9, 4, 3, ranges, off, ids, **kw)
    with pytest.raises(nat.UngxError) as e:
        p.shard_rows()
    assert e.value.status == nat.UNGX_ERR_INVALID_ARG


def test_flat_to_csr():
    flat = np.array([3, 1, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 7, 8, 9], dtype=np.uint32)
    off, cols = nat.flat_to_csr(flat, 3, 3)
    assert off.tolist() == [0, 2, 2, 5]
    assert cols.tolist() == [3, 1, 7, 8, 9]
