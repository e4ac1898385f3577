"""Downstream filtered search on an index built on the device (benchmark configuration 5
at reduced size: the configuration-2 distributions with 30,000 points, 512 queries of
1-2 labels, containment filter, greedy search L = 100, top-10).

The whole index graph is built through the C ABI on the GPU -- intra-group edges by
ungx_exact_knn_graph_device, cross edges by ungx_cross_edges_generate_device,
additional edges by ungx_additional_edges_build, per-point emission by
ungx_graph_csr_device -- and compared with the same graph built by the CPU oracle
(the reference's cross-edge, additional-edge and kNN steps restated).  Both graphs are
then searched by the oracle's restatement of the reference's greedy search and scored
against the filtered brute-force truth: the recall@10 difference must stay within 0.002
(the north-star bar); with identical graphs it is zero.

The second test runs configuration 5 at its full size (1,000,000 points, 10,240
queries; about 30 s on one B200 with 16 host cores, UNGX_CONFIG5_FULL=0 skips it); its
comparison graph takes the cross and additional
edges from the reference's own compiled code (oracle/_ref) and the intra-group rows
from the device, whose seeding is checked bit for bit elsewhere."""
import os
import time

import numpy as np
import pytest

import oracle as O
from filtervectorcode_refactor_b200 import _native as nat
from search_case import knn_config, make_case, oracle_graph, search_recall

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

RECALL_TOLERANCE = 0.002


def device_graph(ctx, case):
    """The index graph built on the device: CSR offsets, columns, group entry points,
    and the kNN seeding's rows (host copy)."""
    n, k, d = case["n"], case["k"], case["Xr"].shape[1]
    G = case["num_groups"]
    ctx.prepare_base_vectors(case["Xr"], n, d, on_device=False)
    try:
        cfg = knn_config()
        d_rows = torch.empty((n, cfg.graph_stride), dtype=torch.int32, device="cuda")
        d_entry = torch.empty((G,), dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        ctx.exact_knn_graph_device(case["group_ranges"][2:], cfg, d_rows.data_ptr(), d_entry.data_ptr())
        torch.cuda.synchronize()
        # [degree, local ids ...] rows -> intra-group CSR over global ids (device tensors)
        deg = d_rows[:, 0].long()
        i_off = torch.zeros(n + 1, dtype=torch.int64, device="cuda")
        i_off[1:] = torch.cumsum(deg, 0)
        mask = torch.arange(cfg.graph_stride - 1, device="cuda")[None, :] < deg[:, None]
        first = torch.from_numpy(case["group_first"][case["group_of"]].astype(np.int64)).cuda()
        i_cols = (d_rows[:, 1:].long() + first[:, None])[mask].to(torch.int32).contiguous()

        prob = nat.Problem(n, d, k, case["group_ranges"], case["out_offsets"], case["out_ids"],
                           route=nat.ROUTE_TENSOR)
        d_ids = torch.empty((n, k), dtype=torch.int32, device="cuda")
        d_dists = torch.empty((n, k), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        ctx.generate_device(prob, d_ids.data_ptr(), d_dists.data_ptr())
        st = ctx.additional_edges(prob, d_ids.data_ptr())
        torch.cuda.synchronize()
        cap = int(i_cols.numel()) + n * k + int(st.edges)
        d_off = torch.empty(n + 1, dtype=torch.int64, device="cuda")
        d_cols = torch.empty(cap, dtype=torch.int32, device="cuda")
        total = ctx.graph_csr_device(n, k, i_off.data_ptr(), i_cols.data_ptr(), d_ids.data_ptr(), True,
                                     d_off.data_ptr(), d_cols.data_ptr(), cap)
        torch.cuda.synchronize()
    finally:
        ctx.release_base_vectors()
    off = d_off.cpu().numpy().view(np.uint64)
    cols = d_cols.cpu().numpy().view(np.uint32)[:total]
    entry = np.zeros(G + 1, dtype=np.uint32)
    entry[1:] = d_entry.cpu().numpy().view(np.uint32)
    return off, cols, entry, d_rows.cpu().numpy().view(np.uint32)


def test_search_recall_on_device_built_index():
    case = make_case(30_000, 512, seed=5)
    with nat.Context(0) as ctx:
        g_off, g_cols, g_entry, _ = device_graph(ctx, case)
    o_off, o_cols, o_entry = oracle_graph(case)
    assert np.array_equal(g_entry, o_entry)
    assert np.array_equal(g_off, o_off)
    assert np.array_equal(g_cols, o_cols)
    r_dev, res_dev, gt = search_recall(case, g_off, g_cols, g_entry)
    r_orc, res_orc, _ = search_recall(case, o_off, o_cols, o_entry)
    print(f"config-5 check: n={case['n']} nq={case['Q'].shape[0]} edges={g_cols.size} "
          f"recall@10 device-built {r_dev:.4f} oracle-built {r_orc:.4f}")
    assert abs(r_dev - r_orc) <= RECALL_TOLERANCE
    assert np.array_equal(res_dev, res_orc)
    assert r_dev > 0.5


@pytest.mark.skipif(os.environ.get("UNGX_CONFIG5_FULL") == "0",
                    reason="full configuration 5 (1M points, 10,240 queries) skipped by UNGX_CONFIG5_FULL=0")
def test_search_recall_full_configuration_5():
    ref = O.reference()
    if ref is None:
        pytest.skip("reference build (oracle/_ref) absent")
    t = time.perf_counter()
    case = make_case(1_000_000, 10_240, seed=0)
    t_case = time.perf_counter() - t
    t = time.perf_counter()
    with nat.Context(0) as ctx:
        g_off, g_cols, g_entry, rows = device_graph(ctx, case)
    t_dev = time.perf_counter() - t
    t = time.perf_counter()
    r_off, r_cols, r_entry = oracle_graph(case, intra_rows=rows, lib=ref)
    t_ref = time.perf_counter() - t
    assert np.array_equal(g_off, r_off)
    assert np.array_equal(g_cols, r_cols)
    assert np.array_equal(g_entry, r_entry)
    t = time.perf_counter()
    truth, _ = ref.filtered_scan(case["Xr"], case["group_first"], case["Q"], case["target_offsets"],
                                 case["target_ids"], case["K"])
    t_truth = time.perf_counter() - t
    r_dev, res_dev, _ = search_recall(case, g_off, g_cols, g_entry, truth)
    r_ref, res_ref, _ = search_recall(case, r_off, r_cols, r_entry, truth)
    print(f"config-5 full: n={case['n']} nq={case['Q'].shape[0]} edges={g_cols.size} recall@10 device-built "
          f"{r_dev:.4f} reference-built {r_ref:.4f}; host set-up {t_case:.1f} s, device graph {t_dev:.1f} s, "
          f"reference graph {t_ref:.1f} s, truth {t_truth:.1f} s")
    assert abs(r_dev - r_ref) <= RECALL_TOLERANCE
    assert np.array_equal(res_dev, res_ref)
