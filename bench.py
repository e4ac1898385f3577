"""Benchmark of the UNG cross-edge build on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--extra-configs 3,4]
                    [--impl ours|reference] [--stage cross|graph]

One step = the cross-edge generate step of UniNavGraph (the seam
build_cross_edges_generate_gpu_optimized) over the whole synthetic workload, through the
library's multi-GPU entry point ungx_cross_edges_build_distributed: build the resident
tensor-core operand from the base vectors already in HBM, run the prefilter, rerank and
rescan kernels on this rank's shard of the work items, and (N > 1) gather every shard's
rows on rank 0 with the library's NCCL send / receive.  The plan (host work that
depends only on the label structure) is made by the first warm-up step and reused.

Headline workload: n = 1,000,000, d = 128, rows
L2-normalised, 30 labels, k = 6.  The same line carries sub-records for configuration 3
(1M x 960, k = 16) and configuration 4 (10M x 96, k = 6), each timed in the same process.
value = algorithmic TFLOP/s = 2 * d * W / step time, W = the number of (source vector,
target vector) pairs over all LNG edges (the reference's dim_ops / d).  Multi-GPU: the
same problem's work items are split across ranks (strong scaling), timed as the max
over ranks.  torch.distributed carries only set-up traffic (the NCCL id, the input
broadcast), barriers and the max over ranks -- nothing inside a timed step.

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
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "UNG cross-edge build TFLOP/s (algorithmic 2*d*W / wall), configs[1]"
# DRAM bytes (read + write) of one tc_kernel launch on the configuration-2 workload, from
# one ncu capture of this build (profiles/tc_kernel_cfg2.txt); other configurations: none.
TC_TRAFFIC_BYTES = {2: 556_360_704 + 202_750_976}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def problem_arrays(label_offsets, labels, source: str = "library") -> dict:
    """Groups, reorder and LNG of the label sets: the library's (source='library') or the
    reference's own TrieIndex build in oracle/_ref (source='reference')."""
    if source == "reference":
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        ref = O.reference()
        impl = ref if ref is not None else O.oracle()
        r = impl.label_graph(label_offsets, labels)
        return dict(num_groups=int(r["num_groups"]), new_to_old=r["new_to_old"], group_ranges=r["group_ranges"],
                    out_offsets=r["out_offsets"], out_ids=r["out_ids"])
    from filtervectorcode_refactor_b200 import _native as nat
    lg = nat.LabelGraph(label_offsets, labels)
    return dict(num_groups=int(lg.num_groups), new_to_old=lg.new_to_old, group_ranges=lg.group_ranges,
                out_offsets=lg.out_offsets, out_ids=lg.out_ids)


def pair_count(pa: dict) -> int:
    """W = sum over LNG edges f -> f' of |f| * |f'|."""
    gr = pa["group_ranges"].reshape(-1, 2).astype(np.int64)
    sizes = gr[:, 1] - gr[:, 0]
    oo = pa["out_offsets"].astype(np.int64)
    G = pa["num_groups"]
    src = np.repeat(np.arange(G + 1), np.diff(oo[:G + 2]))
    return int(np.sum(sizes[src] * sizes[pa["out_ids"].astype(np.int64)]))


def load_workload(cfg: int, seed: int = 0, source: str = "library"):
    from filtervectorcode_refactor_b200 import datasets
    c = datasets.make_config(cfg, seed=seed)
    pa = problem_arrays(c["label_offsets"], c["labels"], source)
    Xr = datasets.reorder_rows(c["X"], pa["new_to_old"])
    del c["X"]
    return c, pa, Xr, pair_count(pa)


def sample_source_groups(pa, budget_pairs: int, rng) -> tuple[np.ndarray, int]:
    """A deterministic stratified sample of source groups whose pair count is about
    budget_pairs (every size bucket represented)."""
    G = pa["num_groups"]
    gr = pa["group_ranges"].reshape(-1, 2).astype(np.int64)
    sizes = gr[:, 1] - gr[:, 0]
    oo = pa["out_offsets"].astype(np.int64)
    src = np.repeat(np.arange(G + 1), np.diff(oo[:G + 2]))
    cost = np.zeros(G + 1, dtype=np.int64)
    np.add.at(cost, src, sizes[src] * sizes[pa["out_ids"].astype(np.int64)])
    cand = np.nonzero(cost > 0)[0]
    order = rng.permutation(cand)
    mask = np.zeros(G + 1, dtype=np.uint8)
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


def cpu_exact_sample(pa, Xr, k, budget_pairs, seed=0, threads=0):
    """Times the reference CPU exact scan on a sample; returns (TFLOP/s, seconds, pairs, kind)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    impl = O.reference()
    kind = "reference"
    if impl is None:
        impl, kind = O.oracle(), "port"
    mask, _ = sample_source_groups(pa, budget_pairs, np.random.default_rng(seed))
    gr = pa["group_ranges"]
    gf = np.concatenate([[0], gr[2::2], [gr[-1]]]).astype(np.uint32)
    t0 = time.perf_counter()
    _, _, pairs = impl.cross_exact(Xr, k, gf, pa["out_offsets"], pa["out_ids"], source_mask=mask, num_threads=threads)
    dt = time.perf_counter() - t0
    return 2.0 * Xr.shape[1] * pairs / dt / 1e12, dt, pairs, kind


def cpu_baseline(pa, Xr, k, W, seconds):
    """The reference's CPU exact scan on a sample of about `seconds` of host work."""
    threads = os.cpu_count() or 1
    _, dt0, p0, _ = cpu_exact_sample(pa, Xr, k, 100_000_000 if Xr.shape[1] <= 128 else 20_000_000, threads=threads)
    budget = int(p0 * seconds / max(dt0, 1e-3))
    rate, dt, pairs, kind = cpu_exact_sample(pa, Xr, k, budget, seed=1, threads=threads)
    return {"value": round(rate, 4), "unit": "TFLOP/s", "cores": threads, "kind": kind,
            "sample": f"{pairs} of W={W} pairs (stratified source groups), {dt:.1f} s, OpenMP dynamic,1"}


class ClockSampler:
    """nvidia-smi samples of one GPU's clocks and throttle reasons during a timed region
    (written to a temporary file)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        fd, self.path = tempfile.mkstemp(prefix=f"ungx_clocks{device}_", suffix=".csv")
        os.close(fd)

    def __enter__(self):
        try:
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
        try:
            os.unlink(self.path)
        except OSError:
            pass
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
    """The reference's CPU exact scan on the headline workload (rank 0 only); groups, reorder
    and LNG from the reference's own TrieIndex build (oracle/_ref)."""
    if rank != 0:
        return
    c, pa, Xr, W = load_workload(args.config, source="reference")
    threads = os.cpu_count() or 1
    # size each step's sample so the whole run takes about 2.5 minutes of CPU time
    per_step_s = min(10.0, max(1.0, 150.0 / (args.steps + args.warmup)))
    rate, dt, pairs, kind = cpu_exact_sample(pa, Xr, c["k"], 200_000_000, threads=threads)
    budget = int(max(1e6, per_step_s * pairs / max(dt, 1e-3)))
    vals = []
    for i in range(args.warmup + args.steps):
        rate, dt, pairs, kind = cpu_exact_sample(pa, Xr, c["k"], budget, seed=i, threads=threads)
        if i >= args.warmup:
            vals.append((rate, dt, pairs))
    value = statistics.median(v[0] for v in vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * statistics.median(v[1] for v in vals), 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": c["name"], "n": c["n"], "d": c["d"], "k": c["k"], "groups": pa["num_groups"],
                   "lng_edges": int(pa["out_ids"].size), "pairs_W": W},
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": threads, "kind": kind,
                         "sample": f"stratified source-group sample, ~{int(statistics.median(v[2] for v in vals))} "
                                   f"of W={W} pairs per step, exact scan (UNG_CROSS_EDGE_IMPL=3), OpenMP dynamic,1"},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


class Ranks:
    """The process group used for set-up, barriers and the max over ranks."""

    def __init__(self, rank, world, local_rank):
        self.rank, self.world, self.local_rank = rank, world, local_rank

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max(self, v: float) -> float:
        if self.world == 1:
            return v
        import torch
        import torch.distributed as dist
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{self.local_rank}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, v: int) -> int:
        if self.world == 1:
            return v
        import torch
        import torch.distributed as dist
        t = torch.tensor([v], dtype=torch.int64, device=f"cuda:{self.local_rank}")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return int(t.item())

    def gather(self, obj):
        if self.world == 1:
            return [obj]
        import torch.distributed as dist
        out = [None] * self.world
        dist.all_gather_object(out, obj)
        return out

    def broadcast_array(self, a: np.ndarray | None, dtype) -> np.ndarray:
        """Rank 0's host array on every rank (over the NCCL process group)."""
        if self.world == 1:
            return a
        import torch
        import torch.distributed as dist
        dev = f"cuda:{self.local_rank}"
        view = {np.uint32: torch.int32, np.uint64: torch.int64, np.float32: torch.float32}[dtype]
        npv = {np.uint32: np.int32, np.uint64: np.int64, np.float32: np.float32}[dtype]
        size = torch.tensor([a.size if self.rank == 0 else 0], dtype=torch.int64, device=dev)
        dist.broadcast(size, 0)
        t = (torch.from_numpy(np.ascontiguousarray(a).view(npv)).to(dev) if self.rank == 0
             else torch.empty(int(size.item()), dtype=view, device=dev))
        dist.broadcast(t, 0)
        return t.cpu().numpy().view(dtype)


def bench_config(args, ranks: Ranks, ctx, cfg: int, steps: int, warmup: int, cpu_seconds: float) -> dict:
    """One configuration through ungx_cross_edges_build_distributed on every rank: the
    device-resident step (value), the host-buffer step (e2e), the per-rank breakdown."""
    import torch
    import torch.distributed as dist
    from filtervectorcode_refactor_b200 import _native as nat
    from filtervectorcode_refactor_b200 import datasets
    rank, world, lr = ranks.rank, ranks.world, ranks.local_rank
    dev = torch.device("cuda", lr)
    c = dict(datasets.CONFIGS[cfg])
    if rank == 0:
        c, pa, Xr, W = load_workload(cfg)
        meta = np.array([Xr.shape[0], Xr.shape[1], c["k"], pa["num_groups"], W], dtype=np.uint64)
    else:
        pa, Xr, meta = {}, None, None
    meta = ranks.broadcast_array(meta, np.uint64)
    n, d, k, G, W = (int(x) for x in meta)
    for key in ("group_ranges", "out_ids"):
        pa[key] = ranks.broadcast_array(pa.get(key), np.uint32)
    pa["out_offsets"] = ranks.broadcast_array(pa.get("out_offsets"), np.uint64)
    pa["num_groups"] = G
    # the base vectors: resident in every GPU's memory (value), and this rank's slice in
    # pinned host memory (e2e)
    if rank == 0:
        X = torch.from_numpy(Xr).to(dev)
    else:
        X = torch.empty((n, d), dtype=torch.float32, device=dev)
    if world > 1:
        dist.broadcast(X, 0)
    a, cnt = nat.dist_slice(n, world, rank)
    slice_h = X[a:a + cnt].cpu().pin_memory()
    prob = nat.Problem(n, d, k, pa["group_ranges"], pa["out_offsets"], pa["out_ids"], route=nat.ROUTE_TENSOR)
    flops_total = 2.0 * d * W
    d_ids = torch.empty(n * k if rank == 0 else 1, dtype=torch.int32, device=dev)
    d_dists = torch.empty(n * k if rank == 0 else 1, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    timings = []
    flags = nat.DIST_DEVICE_VECTORS | nat.DIST_DEVICE_OUTPUT

    def step():
        t = ctx.build_distributed(X.data_ptr(), prob, d_ids.data_ptr(), d_dists.data_ptr(), flags)
        timings.append(t.as_dict())

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    ranks.barrier()
    timings.clear()
    with ClockSampler(lr) as clk:
        torch.cuda.synchronize()
        ranks.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(steps):
            step()  # each call returns after its device work (and the gather) completed
        e.record(stream)
        torch.cuda.synchronize()
        ranks.barrier()
    ms = ranks.max(s.elapsed_time(e))
    ms_step = ms / steps
    launches = ranks.sum(sum(t["gpu_launches"] for t in timings))
    med = lambda key, sub=None: statistics.median((t[sub][key] if sub else t[key]) for t in timings)
    mine = {"tc_kernel_ms": med("tc_kernel_ms", "cross"), "rerank_ms": med("rerank_ms", "cross"),
            "fallback_ms": med("fallback_ms", "cross"), "plan_ms": med("plan_ms", "cross"),
            "prepare_ms": med("prepare_ms"), "gather_ms": med("gather_ms"), "total_ms": med("total_ms"),
            "pairs": timings[-1]["cross"]["pairs"], "rows": timings[-1]["shard_rows"],
            "shard_cost": timings[-1]["shard_cost"], "plan_reused": timings[-1]["plan_reused"],
            "rows_certified": timings[-1]["cross"]["rows_certified"],
            "rows_rescanned": timings[-1]["cross"]["rows_fallback"]}
    per_rank = ranks.gather(mine)
    clocks = clk.summary()

    # ---- end to end through the public C ABI with host buffers: every rank passes its
    # slice of the pinned host vectors; rank 0 receives the whole output in pinned host
    # buffers.  H2D of the slices, NVLink replication, kernels, gather and D2H are inside.
    h_ids = torch.empty(n * k if rank == 0 else 1, dtype=torch.int32).pin_memory()
    h_d = torch.empty(n * k if rank == 0 else 1, dtype=torch.float32).pin_memory()
    sn = slice_h.numpy()
    idn, dn = (h_ids.numpy().view(np.uint32), h_d.numpy()) if rank == 0 else (None, None)
    for _ in range(2):
        ctx.build_distributed(sn, prob, idn, dn)
    ranks.barrier()
    reps = max(3, min(steps, 5))
    t0 = time.perf_counter()
    e2e_t = []
    for _ in range(reps):
        e2e_t.append(ctx.build_distributed(sn, prob, idn, dn).as_dict())
    e2e_ms = ranks.max((time.perf_counter() - t0) * 1e3 / reps)
    e2e = {"value": round(flops_total / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s", "ms_per_step": round(e2e_ms, 3),
           "h2d_bytes_per_step": int(n * d * 4), "d2h_bytes_per_step": int(n * k * 8),
           "upload_ms_rank": round(statistics.median(t["upload_ms"] for t in e2e_t), 3),
           "replicate_ms_rank": round(statistics.median(t["replicate_ms"] for t in e2e_t), 3),
           "d2h_ms_rank0": round(statistics.median(t["d2h_ms"] for t in e2e_t), 3) if rank == 0 else None}
    if rank == 0:
        nonzero = np.count_nonzero(h_ids.numpy() != -1)
        assert nonzero > 0, "the gathered output is empty"

    rec = None
    if rank == 0:
        peak, peak_source = tensor_peak()
        tc_max = max(r["tc_kernel_ms"] for r in per_rank)
        achieved = 2.0 * d * per_rank[0]["pairs"] / (per_rank[0]["tc_kernel_ms"] * 1e-3) / 1e12
        costs = [r["shard_cost"] for r in per_rank]
        rec = {
            "workload": c["name"], "n": n, "d": d, "k": k, "groups": G, "lng_edges": int(pa["out_ids"].size),
            "pairs_W": W, "flops_per_step": flops_total, "steps": steps, "warmup": warmup,
            "ms_per_step": round(ms_step, 4), "value": round(flops_total / (ms_step * 1e-3) / 1e12, 3),
            "wall_s_per_build": round(ms_step / 1e3, 6), "gpu_launches": launches,
            "roofline": {"bound": "tensor", "kernel": "tc_kernel (rank 0)", "achieved": round(achieved, 2),
                         "peak": round(peak, 1), "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                         "peak_source": peak_source, "traffic": TC_TRAFFIC_BYTES.get(cfg) if world == 1 else None},
            "e2e": e2e,
            "per_rank": [{key: (round(v, 4) if isinstance(v, float) else v) for key, v in r.items()}
                         for r in per_rank],
            "imbalance": {"shard_cost_max_over_mean": round(max(costs) / (sum(costs) / len(costs)), 4),
                          "tc_ms_max_over_mean": round(tc_max / statistics.mean(r["tc_kernel_ms"] for r in per_rank),
                                                       4)},
            "clocks": clocks,
        }
        if world == 1 and cpu_seconds > 0:
            rec["cpu_baseline"] = cpu_baseline(pa, Xr, k, W, cpu_seconds)
    del X, d_ids, d_dists, slice_h, h_ids, h_d
    ctx.release_base_vectors()
    torch.cuda.empty_cache()
    ranks.barrier()
    return rec


def run_ours(args, ranks: Ranks):
    import torch
    import torch.distributed as dist
    from filtervectorcode_refactor_b200 import _native as nat

    torch.cuda.set_device(ranks.local_rank)
    ctx = nat.Context(ranks.local_rank)
    if ranks.world > 1:
        cid = np.frombuffer(nat.comm_id_create(), dtype=np.uint8) if ranks.rank == 0 else np.zeros(128, np.uint8)
        t = torch.from_numpy(cid.copy()).to(f"cuda:{ranks.local_rank}")
        dist.broadcast(t, 0)
        ctx.comm_init(bytes(t.cpu().numpy()), ranks.world, ranks.rank)
    head = bench_config(args, ranks, ctx, args.config, args.steps, args.warmup, args.cpu_seconds)
    extra = {}
    for cfg in [int(x) for x in args.extra_configs.split(",") if x.strip()]:
        if cfg == args.config:
            continue
        extra[str(cfg)] = bench_config(args, ranks, ctx, cfg, args.extra_steps, args.warmup, args.extra_cpu_seconds)
    if ranks.world > 1:
        ctx.comm_destroy()
    ctx.close()
    if ranks.rank != 0:
        return
    r0 = head["per_rank"][0]
    line = {
        "metric": METRIC, "value": head["value"], "unit": "TFLOP/s", "n_gpus": ranks.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16+f32",
        "data": "synthetic (seeded, BASELINE configs distributions)",
        "config": {"workload": head["workload"], "n": head["n"], "d": head["d"], "k": head["k"],
                   "groups": head["groups"], "lng_edges": head["lng_edges"], "pairs_W": head["pairs_W"],
                   "flops_per_step": head["flops_per_step"], "wall_s_per_build": head["wall_s_per_build"],
                   "parallelism": f"LNG work-item shards x{ranks.world} (NCCL gather in libungx)",
                   "route": "tcgen05 kind::f16 prefilter (fp16 operand, fp32 accumulate) + exact fp32 rerank",
                   "plan": "made by the first warm-up step, reused (depends on the labels only)",
                   "l2": "inputs larger than L2 (n*d*4 = %d MB base + fp16 operand), no flush"
                         % (head["n"] * head["d"] * 4 >> 20),
                   "rows_certified": r0["rows_certified"], "rows_rescanned": r0["rows_rescanned"]},
        "gpu_launches": head["gpu_launches"],
        "roofline": head["roofline"],
        "cpu_baseline": head.get("cpu_baseline"),
        "e2e": head["e2e"],
        "clocks": head["clocks"],
        "per_rank": head["per_rank"],
        "imbalance": head["imbalance"],
        "configs": extra,
    }
    print(json.dumps(line), flush=True)


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
    c, pa, Xr, W = load_workload(args.config)
    n, d, k = Xr.shape[0], Xr.shape[1], c["k"]
    ctx = nat.Context(0)
    X = torch.from_numpy(Xr).cuda()
    ctx.prepare_base_vectors(X.data_ptr(), n, d, on_device=True)
    gr = pa["group_ranges"].reshape(-1, 2)[1:].astype(np.int64)
    sizes = gr[:, 1] - gr[:, 0]
    sel = np.nonzero((sizes > 64) & (sizes <= 4096))[0]
    ranges = gr[sel].astype(np.uint32).ravel()
    pts = int(sizes[sel].sum())
    pairs = int(np.sum(sizes[sel] * (sizes[sel] - 1)))
    cfg = nat.exact_knn_default_config(64, 32)
    d_graph = torch.empty((max(pts, 1), cfg.graph_stride), dtype=torch.int32, device="cuda")
    knn = {}
    for route_name, route in (("exact", nat.ROUTE_EXACT), ("tensor", nat.ROUTE_TENSOR)):
        cfg.route = route
        for _ in range(args.warmup):
            ctx.exact_knn_graph_device(ranges, cfg, d_graph.data_ptr())
        knn[route_name] = statistics.median(ctx.exact_knn_graph_device(ranges, cfg, d_graph.data_ptr())
                                            for _ in range(max(args.steps, 1)))
        if route_name == "exact":
            exact_rows = d_graph[:pts].clone()
    knn_rejected = ctx.knn_rejected_rows()
    knn_phases = {k: round(v, 3) for k, v in ctx.knn_phase_ms().items()}
    knn_equal = bool(torch.equal(exact_rows, d_graph[:pts]))
    knn_ms = knn["tensor"]
    del exact_rows
    # every group above 64 points, the largest included (the role the reference gives to
    # GNN descent above its exact-batch size): the tensor route, exact and certified
    big = np.nonzero(sizes > 64)[0]
    big_ranges = gr[big].astype(np.uint32).ravel()
    big_pts = int(sizes[big].sum())
    big_pairs = int(np.sum(sizes[big] * (sizes[big] - 1)))
    cfg.route = nat.ROUTE_TENSOR
    g_big = torch.empty((max(big_pts, 1), cfg.graph_stride), dtype=torch.int32, device="cuda")
    ctx.exact_knn_graph_device(big_ranges, cfg, g_big.data_ptr())
    big_ms = statistics.median(ctx.exact_knn_graph_device(big_ranges, cfg, g_big.data_ptr())
                               for _ in range(max(min(args.steps, 3), 1)))
    big_rejected = ctx.knn_rejected_rows()
    big_phases = {k: round(v, 3) for k, v in ctx.knn_phase_ms().items()}
    del g_big
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
    prob = nat.Problem(n, d, k, pa["group_ranges"], pa["out_offsets"], pa["out_ids"], route=nat.ROUTE_AUTO)
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
                        "route": "tcgen05 fp16 self-join prefilter + the reference's distance for 96 candidates",
                        "rows_rejected": int(knn_rejected), "phases_ms": knn_phases,
                        "exact_route_ms": round(knn["exact"], 3),
                        "routes_equal": knn_equal,
                        "tflops_algorithmic": round(2.0 * d * pairs / (knn_ms * 1e-3) / 1e12, 3),
                        "cpu_baseline": {"kind": "port", "cores": os.cpu_count(),
                                         "sample_pairs": int(acc), "seconds": round(cpu_dt, 2),
                                         "tflops": round(2.0 * d * acc / cpu_dt / 1e12, 4)}},
        "knn_seeding_all_groups": {"groups": int(big.size), "points": big_pts, "pairs": big_pairs,
                                   "largest_group": int(sizes[big].max()) if big.size else 0,
                                   "ms": round(big_ms, 3), "rows_rejected": int(big_rejected),
                                   "phases_ms": big_phases,
                                   "tflops_algorithmic": round(2.0 * d * big_pairs / (big_ms * 1e-3) / 1e12, 3)},
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
    ap.add_argument("--config", type=int, default=2, help="headline configuration (BASELINE configs index)")
    ap.add_argument("--extra-configs", default="3,4",
                    help="configurations timed in the same run as sub-records ('' for none)")
    ap.add_argument("--extra-steps", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="CPU work of the headline cpu_baseline sample (seconds on this host)")
    ap.add_argument("--extra-cpu-seconds", type=float, default=6.0,
                    help="CPU work of each sub-record's cpu_baseline sample")
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

        import torch
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, Ranks(rank, world, local_rank))
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
