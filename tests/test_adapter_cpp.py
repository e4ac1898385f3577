"""The C++ adapter (include/ungx_ung_adapter.hpp) as the reference's UniNavGraph would use it.

* It compiles against libungx.so with SearchQueue-shaped stand-in types, and without a
  usable device it reports failure the way the reference's seam does (ok = false plus a
  message) instead of crashing.
* On a B200, oracle/_ref/adapter_check -- the adapter compiled with the reference's own
  headers (search_queue.h, graph.h) and linked with the reference's compiled
  ANNS::SearchQueue -- runs every golden case through the three writeback modes, the
  generate + additional-edge path (materialized[group] lists) and the whole
  build_cross_group_edges step into an ANNS::Graph; every output must equal the
  fixtures made by the reference's compiled code.
"""
import os
import shutil
import subprocess

import numpy as np
import pytest

from conftest import ROOT, have_gpu
from graph_case import expected_merged_graph, local_intra_graph

ADAPTER_CHECK = os.path.join(ROOT, "oracle", "_ref", "adapter_check")

SRC = r"""
#include <cstdio>
#include <utility>
#include <vector>
#include "ungx_ung_adapter.hpp"

// minimal stand-in with the members the adapter uses (reserve, insert, size)
struct Queue {
   std::vector<std::pair<unsigned, float>> v;
   int cap = 0;
   void reserve(int c) { cap = c; }
   void insert(unsigned id, float d) { if ((int)v.size() < cap) v.emplace_back(id, d); }
};

int main() {
   ungx_context *ctx = nullptr;
   int st = ungx_context_create(0, &ctx);
   if (st != UNGX_OK) { std::printf("NO_CONTEXT %d %s\n", st, ungx_last_error(nullptr)); return 0; }
   std::vector<float> X(4 * 2, 0.f);
   for (int i = 0; i < 8; ++i) X[i] = float(i);
   std::vector<std::pair<unsigned, unsigned>> ranges = {{0, 0}, {0, 2}, {2, 4}};
   std::vector<std::vector<unsigned>> lng = {{}, {2}, {}};
   std::vector<Queue> qs;
   auto r = ungx_adapter::generate_cross_edges<Queue, unsigned>(ctx, X.data(), 4, 2, 1, ranges, lng,
                                                               ungx_adapter::Writeback::SearchQueue, &qs,
                                                               nullptr, nullptr);
   std::printf("RESULT %d %zu\n", r.ok ? 1 : 0, qs.size());
   ungx_context_destroy(ctx);
   return 0;
}
"""


def build_probe(tmp_path):
    if shutil.which("g++") is None:
        pytest.skip("no C++ compiler")
    src = tmp_path / "probe.cpp"
    src.write_text(SRC)
    exe = tmp_path / "probe"
    libdir = os.path.join(ROOT, "filtervectorcode_refactor_b200")
    subprocess.run(["g++", "-std=c++17", "-O1", f"-I{ROOT}/include", str(src), "-o", str(exe), f"-L{libdir}",
                    "-lungx", f"-Wl,-rpath,{libdir}"], check=True)
    return exe


def test_adapter_compiles_and_fails_cleanly_without_device(tmp_path):
    if have_gpu():
        pytest.skip("checks the no-device path")
    out = subprocess.run([str(build_probe(tmp_path))], capture_output=True, text=True, check=True).stdout
    assert out.startswith("NO_CONTEXT -6")


def write_case(path, g, intra_off, intra_cols):
    n, d = g["Xr"].shape
    G = g["num_groups"]
    first = g["group_first"].astype(np.int64)
    group_of = np.searchsorted(first[1:], np.arange(n), side="right").astype(np.uint32)
    with open(path, "wb") as f:
        f.write(np.array([n, d, g["k"], G], dtype=np.uint32).tobytes())
        f.write(np.array([g["out_ids"].size, intra_cols.size], dtype=np.uint64).tobytes())
        for a, t in ((g["Xr"], np.float32), (g["group_ranges"], np.uint32), (g["out_offsets"], np.uint64),
                     (g["out_ids"], np.uint32), (intra_off, np.uint64), (intra_cols, np.uint32), (group_of, np.uint32)):
            f.write(np.ascontiguousarray(a, dtype=t).tobytes())


def read_blocks(path):
    raw = open(path, "rb").read()
    out, pos = [], 0
    while pos < len(raw):
        c = int(np.frombuffer(raw, dtype=np.uint64, count=1, offset=pos)[0])
        pos += 8
        out.append(np.frombuffer(raw, dtype=np.uint32, count=c, offset=pos).copy())
        pos += 4 * c
    return out


def test_adapter_check_reports_no_device(tmp_path, golden):
    if have_gpu():
        pytest.skip("checks the no-device path")
    if not os.path.exists(ADAPTER_CHECK):
        pytest.skip("oracle/_ref/adapter_check is not built (the reference tree was absent at build time)")
    intra_off, intra_cols = local_intra_graph(golden, 5)
    write_case(tmp_path / "in.bin", golden, intra_off, intra_cols)
    out = subprocess.run([ADAPTER_CHECK, str(tmp_path / "in.bin"), str(tmp_path / "out.bin")], capture_output=True,
                         text=True, check=True).stdout
    assert out.startswith("NO_CONTEXT -6")


@pytest.mark.gpu
def test_adapter_with_reference_types(tmp_path, golden):
    if not os.path.exists(ADAPTER_CHECK):
        pytest.skip("oracle/_ref/adapter_check is not built (the reference tree was absent at build time)")
    n = golden["Xr"].shape[0]
    k = golden["k"]
    intra_off, intra_cols = local_intra_graph(golden, 5)
    write_case(tmp_path / "in.bin", golden, intra_off, intra_cols)
    r = subprocess.run([ADAPTER_CHECK, str(tmp_path / "in.bin"), str(tmp_path / "out.bin")], capture_output=True,
                       text=True)
    assert r.returncode == 0 and "DONE 0" in r.stdout, r.stdout + r.stderr
    b = read_blocks(tmp_path / "out.bin")
    q_ids, q_d, cap, idv, flat, a_ids, a_d, add_from, add_to, g_off, g_cols = b
    # SearchQueue writeback: ANNS::SearchQueue contents, capacity k (lazy reserve)
    assert np.array_equal(q_ids, golden["ids"])
    assert np.array_equal(q_d, golden["dists"].view(np.uint32))
    assert np.all(cap == k)
    # IdVector and FlatId writebacks
    assert np.array_equal(idv, golden["ids"])
    assert np.array_equal(flat, golden["ids"])
    # generate + additional edges: the same queues and materialized[group] in the reference's order
    assert np.array_equal(a_ids, golden["ids"]) and np.array_equal(a_d, golden["dists"].view(np.uint32))
    assert np.array_equal(add_from, golden["add_from"])
    assert np.array_equal(add_to, golden["add_to"])
    # the whole build_cross_group_edges step into ANNS::Graph
    e_off, e_cols = expected_merged_graph(golden, intra_off, intra_cols, True)
    assert np.array_equal(g_off.astype(np.uint64), e_off)
    assert np.array_equal(g_cols, e_cols)
    assert g_off.size == n + 1
