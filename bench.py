"""Benchmark of the UNG cross-edge build on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl ours|reference]

One step = the cross-edge generate step of UniNavGraph (the seam
build_cross_edges_generate_gpu_optimized) over the whole synthetic workload: build the
resident tensor-core operand from the base vectors already in HBM, plan, run the
kernels, and (N > 1) gather every shard's rows to rank 0 over NCCL.  The workload is
n = 1,000,000, d = 128, rows L2-normalised,
30 labels, k = 6.  value = algorithmic TFLOP/s = 2 * d * W / step time, W = the
number of (source vector, target vector) pairs over all LNG edges (the reference's
dim_ops / d).  Multi-GPU: the same problem's work items are split across ranks
(strong scaling), timed on the device as the max over ranks.

The reference arm (--impl reference) times the reference's own CPU exact scan
(UNG_CROSS_EDGE_IMPL=3; its compiled leaf sources in oracle/_ref, else the oracle's C
restatement) with all host threads on a bounded sample of source groups of the same
workload, reported in the same unit.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "UNG cross-edge build TFLOP/s (algorithmic 2*d*W / wall), configs[1]"
# DRAM bytes (read + write) of one tc_kernel launch on the bench workload, from one ncu
# capture of this build (profiles/tc_kernel_cfg2.txt); other configurations: not captured.
TC_TRAFFIC_BYTES = {2: 556_360_704 + 202_750_976}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def load_workload(cfg: int, seed: int = 0):
    from filtervectorcode_refactor_b200 import _native as nat
    from filtervectorcode_refactor_b200 import datasets
    c = datasets.make_config(cfg, seed=seed)
    lg = nat.LabelGraph(c["label_offsets"], c["labels"])
    Xr = np.ascontiguousarray(c["X"][lg.new_to_old])
    sizes = np.diff(lg.group_ranges.reshape(-1, 2), axis=1)[:, 0].astype(np.int64)
    W = 0
    for f in range(1, lg.num_groups + 1):
        outs = lg.out_ids[lg.out_offsets[f]:lg.out_offsets[f + 1]].astype(np.int64)
        if outs.size:
            W += int(sizes[f]) * int(sizes[outs].sum())
    return c, lg, Xr, W


def sample_source_groups(lg, budget_pairs: int, rng) -> tuple[np.ndarray, int]:
    """A deterministic stratified sample of source groups whose pair count is about
    budget_pairs (every size bucket represented)."""
    gr = lg.group_ranges.reshape(-1, 2).astype(np.int64)
    sizes = gr[:, 1] - gr[:, 0]
    cost = np.zeros(lg.num_groups + 1, dtype=np.int64)
    for f in range(1, lg.num_groups + 1):
        outs = lg.out_ids[lg.out_offsets[f]:lg.out_offsets[f + 1]].astype(np.int64)
        if outs.size and sizes[f]:
            cost[f] = sizes[f] * sizes[outs].sum()
    cand = np.nonzero(cost > 0)[0]
    order = rng.permutation(cand)
    mask = np.zeros(lg.num_groups + 1, dtype=np.uint8)
    total = 0
    buckets = np.floor(np.log2(np.maximum(sizes[order], 1))).astype(int)
    seen = set()
    for f, b in zip(order, buckets):           # one group of every size bucket first
        if b not in seen and total + cost[f] <= 4 * budget_pairs:
            seen.add(b)
            mask[f] = 1
            total += cost[f]
    for f in order:
        if total >= budget_pairs:
            break
        if not mask[f] and total + cost[f] <= 1.5 * budget_pairs:
            mask[f] = 1
            total += cost[f]
    return mask, int(total)


def cpu_exact_sample(lg, Xr, k, budget_pairs, seed=0, threads=0):
    """Times the reference CPU exact scan on a sample; returns (TFLOP/s, seconds, pairs, kind)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    impl = O.reference()
    kind = "reference"
    if impl is None:
        impl, kind = O.oracle(), "port"
    mask, _ = sample_source_groups(lg, budget_pairs, np.random.default_rng(seed))
    gf = np.concatenate([[0], lg.group_ranges[2::2], [lg.group_ranges[-1]]]).astype(np.uint32)
    t0 = time.perf_counter()
    _, _, pairs = impl.cross_exact(Xr, k, gf, lg.out_offsets, lg.out_ids, source_mask=mask, num_threads=threads)
    dt = time.perf_counter() - t0
    return 2.0 * Xr.shape[1] * pairs / dt / 1e12, dt, pairs, kind


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = os.path.join(ROOT, "gpurun_out", f"clocks_rank{device}.csv")

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
            # the timed region starts once nvidia-smi is sampling
            t_end = time.time() + 5.0
            while time.time() < t_end and os.path.getsize(self.path) == 0 and self.proc.poll() is None:
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "samples": len(sm),
                "reasons": sorted(reasons)}


def tensor_peak() -> tuple[float, str]:
    """Dense fp16/bf16 tensor peak of this pool's B200s (TFLOP/s): the driver-measured
    cuBLAS bf16 GEMM burst figure (the prefilter kernel is timed per launch), else the
    pool's earlier measurement."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            v = float(json.load(f)["bf16_tflops"])
        return v, "of measured (MEASURED_PEAKS.json bf16_tflops, burst; fp16 runs at the bf16 rate)"
    except Exception:
        return 1590.0, "of fallback (1.59 PFLOP/s bf16, earlier measurement on this pool)"


def run_reference(args, rank, world):
    if rank != 0:
        return
    c, lg, Xr, W = load_workload(args.config)
    threads = os.cpu_count() or 1
    # size each step's sample so the whole run takes about 2.5 minutes of CPU time
    per_step_s = min(10.0, max(1.0, 150.0 / (args.steps + args.warmup)))
    rate, dt, pairs, kind = cpu_exact_sample(lg, Xr, c["k"], 200_000_000, threads=threads)
    budget = int(max(1e6, per_step_s * pairs / max(dt, 1e-3)))
    vals = []
    for i in range(args.warmup + args.steps):
        rate, dt, pairs, kind = cpu_exact_sample(lg, Xr, c["k"], budget, seed=i, threads=threads)
        if i >= args.warmup:
            vals.append((rate, dt, pairs))
    value = statistics.median(v[0] for v in vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * statistics.median(v[1] for v in vals), 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": c["name"], "n": c["n"], "d": c["d"], "k": c["k"], "pairs_W": W},
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": threads, "kind": kind,
                         "sample": f"stratified source-group sample, ~{int(statistics.median(v[2] for v in vals))} "
                                   f"of W={W} pairs per step, exact scan (UNG_CROSS_EDGE_IMPL=3), OpenMP dynamic,1"},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from filtervectorcode_refactor_b200 import _native as nat

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    c, lg, Xr, W = load_workload(args.config)
    n, d, k = Xr.shape[0], Xr.shape[1], c["k"]
    flops_total = 2.0 * d * W
    ctx = nat.Context(local_rank)
    prob = nat.Problem(n, d, k, lg.group_ranges, lg.out_offsets, lg.out_ids, route=nat.ROUTE_TENSOR,
                       shard_rank=rank, shard_count=world)
    own_rows = torch.from_numpy(prob.shard_rows().astype(np.int64)).to(dev)
    X = torch.from_numpy(Xr).to(dev)
    d_ids = torch.empty((n, k), dtype=torch.int32, device=dev)
    d_dists = torch.empty((n, k), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    counts = None
    if world > 1:
        cnt = torch.tensor([own_rows.numel()], device=dev)
        allc = [torch.zeros_like(cnt) for _ in range(world)]
        dist.all_gather(allc, cnt)
        counts = [int(x.item()) for x in allc]
        pad = max(counts)
        allrows = [torch.zeros(pad, dtype=torch.int64, device=dev) for _ in range(world)]
        rows_p = torch.zeros(pad, dtype=torch.int64, device=dev)
        rows_p[:own_rows.numel()] = own_rows
        dist.all_gather(allrows, rows_p)
        gbuf = [torch.empty((pad, 2 * k), dtype=torch.int32, device=dev) for _ in range(world)]
        full_ids = torch.empty((n, k), dtype=torch.int32, device=dev)
        full_d = torch.empty((n, k), dtype=torch.float32, device=dev)
    timings = []

    def step():
        ctx.prepare_base_vectors(X.data_ptr(), n, d, on_device=True)
        t = ctx.generate_device(prob, d_ids.data_ptr(), d_dists.data_ptr(), stream.cuda_stream)
        timings.append(t.as_dict())
        if world > 1:
            # gather every shard's rows (ids + distance bits) to all ranks over NCCL
            mine = torch.zeros((max(counts), 2 * k), dtype=torch.int32, device=dev)
            mine[:own_rows.numel(), :k] = d_ids[own_rows]
            mine[:own_rows.numel(), k:] = d_dists[own_rows].view(torch.int32)
            dist.all_gather(gbuf, mine)
            if rank == 0:
                for r in range(world):
                    rr = allrows[r][:counts[r]]
                    full_ids[rr] = gbuf[r][:counts[r], :k]
                    full_d[rr] = gbuf[r][:counts[r], k:].view(torch.float32)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    timings.clear()
    with ClockSampler(local_rank) as clk:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(args.steps):
            step()
        e.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = s.elapsed_time(e)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = flops_total / (ms_step * 1e-3) / 1e12
    tc_ms = statistics.median(t["tc_kernel_ms"] for t in timings)
    shard_pairs = timings[-1]["pairs"]
    launches = sum(t["gpu_launches"] + 3 for t in timings)  # +3: the operand-build kernels of prepare
    fallback_rows = timings[-1]["rows_fallback"]
    certified_rows = timings[-1]["rows_certified"]

    # ---- end to end through the public C ABI with host buffers: every rank uploads the
    # pinned host vectors, computes its shard and copies its rows back to its host
    # buffers (ungx_cross_edges_build); the slowest rank's wall time counts.
    Xh = torch.from_numpy(Xr).pin_memory()
    h_ids = torch.empty(n * k, dtype=torch.int32).pin_memory()
    h_d = torch.empty(n * k, dtype=torch.float32).pin_memory()
    Xn, idn, dn = Xh.numpy(), h_ids.numpy().view(np.uint32), h_d.numpy()
    for _ in range(2):
        ctx.build(Xn, prob, idn, dn)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    reps = max(2, min(args.steps, 5))
    for _ in range(reps):
        ctx.build(Xn, prob, idn, dn)
    e2e_ms = (time.perf_counter() - t0) * 1e3 / reps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    plan_bytes = lg.group_ranges.nbytes + lg.out_offsets.nbytes + lg.out_ids.nbytes
    e2e = {"value": round(flops_total / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
           "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": int(world * (Xr.nbytes + plan_bytes)),
           "d2h_bytes_per_step": int(n * k * 8)}

    if rank == 0:
        peak, peak_source = tensor_peak()
        achieved = 2.0 * d * shard_pairs / (tc_ms * 1e-3) / 1e12
        threads = os.cpu_count() or 1
        _, dt0, p0, _ = cpu_exact_sample(lg, Xr, k, 200_000_000, threads=threads)
        budget = int(p0 * args.cpu_seconds / max(dt0, 1e-3))
        cpu_rate, cpu_dt, cpu_pairs, kind = cpu_exact_sample(lg, Xr, k, budget, seed=1, threads=threads)
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16+f32",
            "data": "synthetic (seeded, BASELINE configs[1] distributions)",
            "config": {"workload": c["name"], "n": n, "d": d, "k": k, "groups": int(lg.num_groups),
                       "lng_edges": int(lg.out_ids.size), "pairs_W": int(W), "flops_per_step": flops_total,
                       "wall_s_per_build": round(ms_step / 1e3, 6), "parallelism": f"item-shards x{world}",
                       "route": "tcgen05 kind::f16 prefilter (fp16 operand, fp32 accumulate) + exact fp32 rerank",
                       "l2": "inputs larger than L2 (n*d*4 = %d MB base + fp16 operand), no flush" % (Xr.nbytes >> 20),
                       "rows_certified": int(certified_rows), "rows_rescanned": int(fallback_rows)},
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor", "kernel": "tc_kernel", "achieved": round(achieved, 2),
                         "peak": round(peak, 1), "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                         "peak_source": peak_source,
                         "traffic": TC_TRAFFIC_BYTES.get(args.config)},
            "cpu_baseline": {"value": round(cpu_rate, 4), "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": kind,
                             "sample": f"{cpu_pairs} of W={W} pairs (stratified source groups), {cpu_dt:.1f} s"},
            "e2e": e2e,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    ctx.close()


def run_graph_stages(args):
    """--stage graph (one GPU): the path's graph stages after the cross edges, each timed
    on the device over the configuration's synthetic workload:
      * exact kNN seeding of the groups in the reference's adaptive exact range
        (65 .. 4096 points; K = 64, degree 32, make_fast_exact_batch_config defaults);
      * additional edges (exact variant) from the cross-edge output;
      * whole-graph CSR emission (kNN rows as intra edges + cross + additional)."""
    import torch
    from filtervectorcode_refactor_b200 import _native as nat
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    torch.cuda.set_device(0)
    c, lg, Xr, W = load_workload(args.config)
    n, d, k = Xr.shape[0], Xr.shape[1], c["k"]
    ctx = nat.Context(0)
    X = torch.from_numpy(Xr).cuda()
    ctx.prepare_base_vectors(X.data_ptr(), n, d, on_device=True)
    gr = lg.group_ranges.reshape(-1, 2)[1:].astype(np.int64)
    sizes = gr[:, 1] - gr[:, 0]
    sel = np.nonzero((sizes > 64) & (sizes <= 4096))[0]
    ranges = gr[sel].astype(np.uint32).ravel()
    pts = int(sizes[sel].sum())
    pairs = int(np.sum(sizes[sel] * (sizes[sel] - 1)))
    cfg = nat.exact_knn_default_config(64, 32)
    d_graph = torch.empty((max(pts, 1), cfg.graph_stride), dtype=torch.int32, device="cuda")
    for _ in range(args.warmup):
        ctx.exact_knn_graph_device(ranges, cfg, d_graph.data_ptr())
    knn_ms = statistics.median(ctx.exact_knn_graph_device(ranges, cfg, d_graph.data_ptr())
                               for _ in range(max(args.steps, 1)))
    # CPU: the oracle restatement (the reference's seeding cannot be built) on a group sample
    rng = np.random.default_rng(0)
    order = rng.permutation(sel.size)
    take, acc = [], 0
    budget = 2e8 * max(args.cpu_seconds, 1.0) / 15.0
    for i in order:
        take.append(sel[i])
        acc += int(sizes[sel[i]] * (sizes[sel[i]] - 1))
        if acc > budget:
            break
    sr = gr[np.sort(np.array(take, dtype=np.int64))].astype(np.uint32).ravel()
    t0 = time.perf_counter()
    O.oracle().exact_knn_graph(Xr, sr, 64, 32, 24, 1, 0, 0, 33)
    cpu_dt = time.perf_counter() - t0
    # cross edges on the device, then additional edges and the CSR
    prob = nat.Problem(n, d, k, lg.group_ranges, lg.out_offsets, lg.out_ids, route=nat.ROUTE_AUTO)
    d_ids = torch.empty((n, k), dtype=torch.int32, device="cuda")
    d_dists = torch.empty((n, k), dtype=torch.float32, device="cuda")
    ctx.generate_device(prob, d_ids.data_ptr(), d_dists.data_ptr())
    torch.cuda.synchronize()
    add = [ctx.additional_edges(prob, d_ids.data_ptr()) for _ in range(max(args.warmup, 1) + 1)][-1]
    # intra edges = the kNN rows of the seeded groups (global ids), other points none
    g = d_graph[:pts].cpu().numpy().view(np.uint32)
    deg = np.zeros(n, dtype=np.int64)
    rows = np.concatenate([np.arange(a, b) for a, b in gr[sel]]) if sel.size else np.zeros(0, np.int64)
    firsts = np.concatenate([np.full(b - a, a) for a, b in gr[sel]]) if sel.size else np.zeros(0, np.int64)
    deg[rows] = g[:, 0]
    intra_off = np.zeros(n + 1, dtype=np.uint64)
    intra_off[1:] = np.cumsum(deg)
    cols = np.zeros(max(int(intra_off[-1]), 1), dtype=np.uint32)
    if rows.size:  # rows ascend, so the row-major selection lands in CSR order
        keep = np.arange(g.shape[1] - 1)[None, :] < g[:, :1].astype(np.int64)
        cols[:int(intra_off[-1])] = (g[:, 1:].astype(np.int64) + firsts[:, None])[keep].astype(np.uint32)
    d_io = torch.from_numpy(intra_off.view(np.int64)).cuda()
    d_ic = torch.from_numpy(cols.view(np.int32)).cuda()
    cap = int(intra_off[-1]) + n * k + int(add.edges)
    d_off = torch.empty(n + 1, dtype=torch.int64, device="cuda")
    d_cols = torch.empty(max(cap, 1), dtype=torch.int32, device="cuda")
    csr = []
    for i in range(max(args.warmup, 1) + max(args.steps, 1)):
        t1 = time.perf_counter()
        total = ctx.graph_csr_device(n, k, d_io.data_ptr(), d_ic.data_ptr(), d_ids.data_ptr(), True,
                                     d_off.data_ptr(), d_cols.data_ptr(), cap)
        csr.append((time.perf_counter() - t1) * 1e3)
    csr_ms = statistics.median(csr[max(args.warmup, 1):])
    csr_bytes = (n + 1) * 8 * 2 + n * k * 4 + int(intra_off[-1]) * 4 * 2 + int(add.edges) * 4 * 2 + total * 4
    line = {
        "metric": "UNG graph stages after the cross edges (exact kNN seeding, additional edges, CSR emission)",
        "config": {"workload": c["name"], "n": n, "d": d, "k": k},
        "knn_seeding": {"groups": int(sel.size), "points": pts, "pairs": pairs, "ms": round(knn_ms, 3),
                        "tflops_algorithmic": round(2.0 * d * pairs / (knn_ms * 1e-3) / 1e12, 3),
                        "cpu_baseline": {"kind": "port", "cores": os.cpu_count(),
                                         "sample_pairs": int(acc), "seconds": round(cpu_dt, 2),
                                         "tflops": round(2.0 * d * acc / cpu_dt / 1e12, 4)}},
        "additional_edges": {"missing_group_edges": int(add.missing_group_edges),
                             "query_vectors": int(add.query_vectors), "edges": int(add.edges),
                             "ms_wall": round(add.ms, 3)},
        "csr_emission": {"columns": int(total), "ms_wall": round(csr_ms, 3),
                         "gbs_algorithmic": round(csr_bytes / (csr_ms * 1e-3) / 1e9, 1)},
    }
    print(json.dumps(line), flush=True)
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="CPU work of the cpu_baseline sample (seconds on this host)")
    ap.add_argument("--stage", default="cross", choices=["cross", "graph"],
                    help="cross: the cross-edge build (the benchmark line); graph: the later graph stages")
    args = ap.parse_args()
    if args.stage == "graph":
        run_graph_stages(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
