"""ctypes binding of the in-tree C ABI library ``libungx.so`` (declared in include/ungx.h).

There is no fallback: if the shared library is missing, importing this module raises
``ImportError`` naming the build command.  Every call checks the returned status and
raises :class:`UngxError` with the library's message.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_double, c_int, c_uint8, c_uint32, c_uint64, c_void_p

import numpy as np

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libungx.so")

UNGX_OK = 0
UNGX_ERR_INVALID_ARG = -1
UNGX_ERR_OOM = -2
UNGX_ERR_CUDA = -3
UNGX_ERR_TIMEOUT = -4
UNGX_ERR_ABORTED = -5
UNGX_ERR_NO_DEVICE = -6
UNGX_ERR_STATE = -7

ROUTE_AUTO = 0
ROUTE_TENSOR = 1
ROUTE_EXACT = 2

EMPTY_ID = 0xFFFFFFFF

INJECT_NONE = 0
INJECT_WITHHOLD_WORK = 1


class UngxError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"ungx status {status}: {message}")
        self.status = status


class CrossEdgeTiming(ctypes.Structure):
    """Layout of ``ungx_cross_edge_timing``."""

    _fields_ = [
        ("generate_ms", c_double),
        ("gpu_h2d_ms", c_double),
        ("gpu_kernel_ms", c_double),
        ("gpu_d2h_ms", c_double),
        ("plan_ms", c_double),
        ("prepare_ms", c_double),
        ("tc_kernel_ms", c_double),
        ("rerank_ms", c_double),
        ("fallback_ms", c_double),
        ("pairs", c_uint64),
        ("rows_certified", c_uint64),
        ("rows_fallback", c_uint64),
        ("route_used", c_uint32),
        ("gpu_launches", c_uint32),
        ("passes", c_uint32),
        ("reserved", c_uint32),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_ if name != "reserved"}


class CrossEdgeProblem(ctypes.Structure):
    """Layout of ``ungx_cross_edge_problem``."""

    _fields_ = [
        ("num_points", c_uint32),
        ("dim", c_uint32),
        ("topk", c_uint32),
        ("num_groups", c_uint32),
        ("group_ranges", POINTER(c_uint32)),
        ("lng_out_offsets", POINTER(c_uint64)),
        ("lng_out_ids", POINTER(c_uint32)),
        ("skip_source_group", POINTER(c_uint8)),
        ("route", c_uint32),
        ("shard_rank", c_uint32),
        ("shard_count", c_uint32),
    ]


class AdditionalStats(ctypes.Structure):
    """Layout of ``ungx_additional_stats``."""

    _fields_ = [
        ("missing_group_edges", c_uint64),
        ("query_vectors", c_uint64),
        ("edges", c_uint64),
        ("ms", c_double),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class CrossGroupStats(ctypes.Structure):
    """Layout of ``ungx_cross_group_stats``."""

    _fields_ = [
        ("cross", CrossEdgeTiming),
        ("additional", AdditionalStats),
        ("cross_edges", c_uint64),
        ("num_cols", c_uint64),
        ("merge_ms", c_double),
        ("total_ms", c_double),
    ]


class DistTiming(ctypes.Structure):
    """Layout of ``ungx_dist_timing``."""

    _fields_ = [
        ("cross", CrossEdgeTiming),
        ("upload_ms", c_double),
        ("replicate_ms", c_double),
        ("prepare_ms", c_double),
        ("gather_ms", c_double),
        ("d2h_ms", c_double),
        ("total_ms", c_double),
        ("shard_rows", c_uint64),
        ("shard_cost", c_uint64),
        ("shard_cost_max", c_uint64),
        ("shard_cost_total", c_uint64),
        ("world_size", c_uint32),
        ("rank", c_uint32),
        ("plan_reused", c_uint32),
        ("gpu_launches", c_uint32),
    ]

    def as_dict(self) -> dict:
        d = {name: getattr(self, name) for name, _ in self._fields_ if name != "cross"}
        d["cross"] = self.cross.as_dict()
        return d


class CommId(ctypes.Structure):
    """Layout of ``ungx_comm_id`` (an NCCL unique id)."""

    _fields_ = [("internal", ctypes.c_char * 128)]


DIST_DEVICE_VECTORS = 1
DIST_DEVICE_OUTPUT = 2

BUILD_ADDITIONAL = 1
BUILD_INTRA_LOCAL_IDS = 2
BUILD_VECTORS_ON_DEVICE = 4


class ExactKnnConfig(ctypes.Structure):
    """Layout of ``ungx_exact_knn_config``."""

    _fields_ = [
        ("candidate_k", c_uint32),
        ("final_degree", c_uint32),
        ("head_keep", c_uint32),
        ("anchor_tail", c_uint32),
        ("anchor_slots", c_uint32),
        ("bidir_anchor", c_uint32),
        ("graph_stride", c_uint32),
        ("route", c_uint32),
    ]


# (name, restype, argtypes) of every exported function, in include/ungx.h order.
_SIGNATURES = [
    ("ungx_context_create", c_int, [c_int, POINTER(c_void_p)]),
    ("ungx_context_destroy", c_int, [c_void_p]),
    ("ungx_last_error", c_char_p, [c_void_p]),
    ("ungx_status_string", c_char_p, [c_int]),
    ("ungx_set_timeout_ms", c_int, [c_void_p, c_uint32]),
    ("ungx_set_device_wait_limit_ns", c_int, [c_void_p, c_uint64]),
    ("ungx_set_fault_injection", c_int, [c_void_p, c_uint32]),
    ("ungx_set_device_memory_limit", c_int, [c_void_p, c_uint64]),
    ("ungx_resident_bytes", c_uint64, [c_uint32, c_uint32, c_uint32]),
    ("ungx_prepare_base_vectors", c_int, [c_void_p, c_void_p, c_uint32, c_uint32, c_int]),
    ("ungx_release_base_vectors", c_int, [c_void_p]),
    ("ungx_cross_edges_generate", c_int,
     [c_void_p, POINTER(CrossEdgeProblem), c_void_p, c_void_p, POINTER(CrossEdgeTiming)]),
    ("ungx_cross_edges_generate_device", c_int,
     [c_void_p, POINTER(CrossEdgeProblem), c_void_p, c_void_p, c_void_p, POINTER(CrossEdgeTiming)]),
    ("ungx_cross_edges_build", c_int,
     [c_void_p, c_void_p, POINTER(CrossEdgeProblem), c_void_p, c_void_p, POINTER(CrossEdgeTiming)]),
    ("ungx_cross_edges_exact_noalloc", c_int,
     [POINTER(CrossEdgeProblem), c_void_p, c_void_p, c_void_p, c_void_p]),
    ("ungx_shard_rows", c_int, [POINTER(CrossEdgeProblem), c_void_p, POINTER(c_uint64)]),
    ("ungx_comm_id_create", c_int, [POINTER(CommId)]),
    ("ungx_comm_init", c_int, [c_void_p, POINTER(CommId), c_int, c_int]),
    ("ungx_comm_destroy", c_int, [c_void_p]),
    ("ungx_dist_slice", c_int, [c_uint32, c_uint32, c_uint32, POINTER(c_uint32), POINTER(c_uint32)]),
    ("ungx_cross_edges_build_distributed", c_int,
     [c_void_p, c_void_p, c_uint32, POINTER(CrossEdgeProblem), c_void_p, c_void_p, POINTER(DistTiming)]),
    ("ungx_label_graph_build", c_int, [c_uint32, c_void_p, c_void_p, c_int, POINTER(c_void_p)]),
    ("ungx_label_graph_destroy", c_int, [c_void_p]),
    ("ungx_label_graph_num_groups", c_uint32, [c_void_p]),
    ("ungx_label_graph_num_edges", c_uint64, [c_void_p]),
    ("ungx_label_graph_copy_groups", c_int, [c_void_p, c_void_p, c_void_p]),
    ("ungx_label_graph_copy_out_neighbors", c_int, [c_void_p, c_void_p, c_void_p]),
    ("ungx_label_graph_copy_in_neighbors", c_int, [c_void_p, c_void_p, c_void_p]),
    ("ungx_label_graph_num_set_labels", c_uint64, [c_void_p]),
    ("ungx_label_graph_copy_label_sets", c_int, [c_void_p, c_void_p, c_void_p]),
    ("ungx_flat_to_csr", c_int, [c_void_p, c_uint32, c_uint32, c_void_p, c_void_p]),
    ("ungx_graph_save_text", c_int, [c_char_p, c_uint32, c_void_p, c_void_p]),
    ("ungx_additional_edges_build", c_int,
     [c_void_p, POINTER(CrossEdgeProblem), c_void_p, c_void_p, POINTER(AdditionalStats)]),
    ("ungx_additional_edges_copy", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    ("ungx_graph_csr_device", c_int,
     [c_void_p, c_uint32, c_uint32, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_uint64,
      POINTER(c_uint64), c_void_p]),
    ("ungx_build_cross_group_edges", c_int,
     [c_void_p, c_void_p, POINTER(CrossEdgeProblem), c_void_p, c_void_p, c_uint32, c_void_p, c_void_p,
      POINTER(CrossGroupStats)]),
    ("ungx_graph_copy", c_int, [c_void_p, c_void_p, c_void_p]),
    ("ungx_exact_knn_default_config", None, [c_uint32, c_uint32, POINTER(ExactKnnConfig)]),
    ("ungx_exact_knn_rejected_rows", c_uint64, [c_void_p]),
    ("ungx_exact_knn_phase_ms", None, [c_void_p, POINTER(c_double)]),
    ("ungx_exact_knn_graph_device", c_int,
     [c_void_p, c_uint32, c_void_p, POINTER(ExactKnnConfig), c_void_p, c_void_p, c_void_p, POINTER(c_double)]),
]

EXPORTED = [name for name, _, _ in _SIGNATURES]


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C filtervectorcode_refactor_b200/csrc` "
            "or `python -c 'import __graft_entry__ as g; g.build()'` (there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, res, args in _SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def _ptr(a: np.ndarray | None) -> int | None:
    return None if a is None else a.ctypes.data


def check(status: int, ctx: int | None = None) -> None:
    if status != UNGX_OK:
        msg = lib.ungx_last_error(ctx)
        raise UngxError(status, msg.decode() if msg else lib.ungx_status_string(status).decode())


class LabelGraph:
    """Grouping + reorder + LNG computed by the library (owning wrapper)."""

    def __init__(self, label_offsets: np.ndarray, labels: np.ndarray, num_threads: int = 0):
        label_offsets = np.ascontiguousarray(label_offsets, dtype=np.uint64)
        labels = np.ascontiguousarray(labels, dtype=np.uint32)
        n = label_offsets.shape[0] - 1
        h = c_void_p()
        check(lib.ungx_label_graph_build(n, _ptr(label_offsets), _ptr(labels) if labels.size else None,
                                         num_threads, ctypes.byref(h)))
        self._h = h
        self.num_points = n
        self.num_groups = int(lib.ungx_label_graph_num_groups(h))
        G = self.num_groups
        self.new_to_old = np.empty(n, dtype=np.uint32)
        self.group_ranges = np.empty(2 * (G + 1), dtype=np.uint32)
        check(lib.ungx_label_graph_copy_groups(h, _ptr(self.new_to_old), _ptr(self.group_ranges)))
        ne = int(lib.ungx_label_graph_num_edges(h))
        self.out_offsets = np.empty(G + 2, dtype=np.uint64)
        self.out_ids = np.empty(max(ne, 1), dtype=np.uint32)[:ne]
        check(lib.ungx_label_graph_copy_out_neighbors(h, _ptr(self.out_offsets), _ptr(self.out_ids)))
        self.in_offsets = np.empty(G + 2, dtype=np.uint64)
        self.in_ids = np.empty(max(ne, 1), dtype=np.uint32)[:ne]
        check(lib.ungx_label_graph_copy_in_neighbors(h, _ptr(self.in_offsets), _ptr(self.in_ids)))
        nl = int(lib.ungx_label_graph_num_set_labels(h))
        self.set_offsets = np.empty(G + 2, dtype=np.uint64)
        self.set_labels = np.empty(max(nl, 1), dtype=np.uint32)[:nl]
        check(lib.ungx_label_graph_copy_label_sets(h, _ptr(self.set_offsets), _ptr(self.set_labels)))

    def close(self) -> None:
        if self._h:
            lib.ungx_label_graph_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Problem:
    """Keeps the arrays a ``CrossEdgeProblem`` points at alive."""

    def __init__(self, num_points: int, dim: int, topk: int, group_ranges: np.ndarray,
                 out_offsets: np.ndarray, out_ids: np.ndarray, skip_source_group: np.ndarray | None = None,
                 route: int = ROUTE_AUTO, shard_rank: int = 0, shard_count: int = 1):
        self.group_ranges = np.ascontiguousarray(group_ranges, dtype=np.uint32)
        self.out_offsets = np.ascontiguousarray(out_offsets, dtype=np.uint64)
        self.out_ids = np.ascontiguousarray(out_ids, dtype=np.uint32)
        if self.out_ids.size == 0:
            self.out_ids = np.zeros(1, dtype=np.uint32)
        self.skip = None if skip_source_group is None else np.ascontiguousarray(skip_source_group, dtype=np.uint8)
        G = self.group_ranges.shape[0] // 2 - 1
        self.c = CrossEdgeProblem(
            num_points, dim, topk, G,
            self.group_ranges.ctypes.data_as(POINTER(c_uint32)),
            self.out_offsets.ctypes.data_as(POINTER(c_uint64)),
            self.out_ids.ctypes.data_as(POINTER(c_uint32)),
            None if self.skip is None else self.skip.ctypes.data_as(POINTER(c_uint8)),
            route, shard_rank, shard_count)

    def shard_rows(self) -> np.ndarray:
        cnt = c_uint64()
        check(lib.ungx_shard_rows(ctypes.byref(self.c), None, ctypes.byref(cnt)))
        rows = np.empty(max(cnt.value, 1), dtype=np.uint32)
        check(lib.ungx_shard_rows(ctypes.byref(self.c), _ptr(rows), ctypes.byref(cnt)))
        return rows[:cnt.value]


class Context:
    """One device context (``ungx_context``)."""

    def __init__(self, device: int = 0):
        h = c_void_p()
        check(lib.ungx_context_create(device, ctypes.byref(h)))
        self.h = h
        self.device = device

    def close(self) -> None:
        if self.h:
            lib.ungx_context_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_timeout_ms(self, ms: int) -> None:
        check(lib.ungx_set_timeout_ms(self.h, ms), self.h)

    def set_device_wait_limit_ns(self, ns: int) -> None:
        check(lib.ungx_set_device_wait_limit_ns(self.h, ns), self.h)

    def set_device_memory_limit(self, nbytes: int) -> None:
        """Device budget of build(); 0 = the free device memory.  Above it, build() takes
        the capacity path (passes over pairs of row slices)."""
        check(lib.ungx_set_device_memory_limit(self.h, nbytes), self.h)

    def set_fault_injection(self, flags: int) -> None:
        check(lib.ungx_set_fault_injection(self.h, flags), self.h)

    def prepare_base_vectors(self, vectors, num_points: int, dim: int, on_device: bool) -> None:
        """``vectors`` is a host numpy array, or (on_device=True) an integer device pointer."""
        ptr = vectors if on_device else _ptr(vectors)
        check(lib.ungx_prepare_base_vectors(self.h, ptr, num_points, dim, int(on_device)), self.h)

    def release_base_vectors(self) -> None:
        check(lib.ungx_release_base_vectors(self.h), self.h)

    def generate(self, problem: Problem, out_ids: np.ndarray, out_dists: np.ndarray | None) -> CrossEdgeTiming:
        t = CrossEdgeTiming()
        check(lib.ungx_cross_edges_generate(self.h, ctypes.byref(problem.c), _ptr(out_ids), _ptr(out_dists),
                                            ctypes.byref(t)), self.h)
        return t

    def generate_device(self, problem: Problem, d_ids: int, d_dists: int | None, stream: int | None = None
                        ) -> CrossEdgeTiming:
        t = CrossEdgeTiming()
        check(lib.ungx_cross_edges_generate_device(self.h, ctypes.byref(problem.c), d_ids, d_dists, stream,
                                                   ctypes.byref(t)), self.h)
        return t

    def build(self, vectors: np.ndarray, problem: Problem, out_ids: np.ndarray, out_dists: np.ndarray | None
              ) -> CrossEdgeTiming:
        t = CrossEdgeTiming()
        check(lib.ungx_cross_edges_build(self.h, _ptr(vectors), ctypes.byref(problem.c), _ptr(out_ids),
                                         _ptr(out_dists), ctypes.byref(t)), self.h)
        return t


    def comm_init(self, comm_id: bytes, world_size: int, rank: int) -> None:
        """ungx_comm_init: join the NCCL communicator of ``comm_id`` (from comm_id_create)."""
        if len(comm_id) != ctypes.sizeof(CommId):
            raise ValueError("a communicator id has 128 bytes")
        cid = CommId()
        ctypes.memmove(ctypes.addressof(cid), comm_id, len(comm_id))
        check(lib.ungx_comm_init(self.h, ctypes.byref(cid), world_size, rank), self.h)

    def comm_destroy(self) -> None:
        check(lib.ungx_comm_destroy(self.h), self.h)

    def build_distributed(self, vectors, problem: Problem, out_ids, out_dists, flags: int = 0) -> DistTiming:
        """ungx_cross_edges_build_distributed.  ``vectors``: this rank's slice (host array,
        rows of dist_slice), or an integer device pointer to the whole matrix with
        DIST_DEVICE_VECTORS.  ``out_ids`` / ``out_dists``: host arrays, or integer device
        pointers with DIST_DEVICE_OUTPUT (rank 0 only; other ranks may pass None)."""
        t = DistTiming()
        vp = vectors if (flags & DIST_DEVICE_VECTORS) else _ptr(vectors)
        if flags & DIST_DEVICE_OUTPUT:
            oi, od = out_ids, out_dists
        else:
            oi, od = _ptr(out_ids), _ptr(out_dists)
        check(lib.ungx_cross_edges_build_distributed(self.h, vp, flags, ctypes.byref(problem.c), oi, od,
                                                     ctypes.byref(t)), self.h)
        return t

    def additional_edges(self, problem: Problem, d_cross_ids: int, stream: int | None = None) -> AdditionalStats:
        """ungx_additional_edges_build on a device cross-edge output [n x k]."""
        st = AdditionalStats()
        check(lib.ungx_additional_edges_build(self.h, ctypes.byref(problem.c), d_cross_ids, stream,
                                              ctypes.byref(st)), self.h)
        return st

    def additional_edges_copy(self, num_points: int, num_edges: int):
        """(from_ids, to_ids, point_offsets, point_cols) of the last additional-edge build."""
        src = np.empty(max(num_edges, 1), dtype=np.uint32)
        dst = np.empty(max(num_edges, 1), dtype=np.uint32)
        off = np.empty(num_points + 1, dtype=np.uint64)
        cols = np.empty(max(num_edges, 1), dtype=np.uint32)
        check(lib.ungx_additional_edges_copy(self.h, _ptr(src), _ptr(dst), _ptr(off), _ptr(cols)), self.h)
        return src[:num_edges], dst[:num_edges], off, cols[:num_edges]

    def build_cross_group_edges(self, vectors, problem: Problem, intra_offsets: np.ndarray | None = None,
                                intra_cols: np.ndarray | None = None, flags: int = BUILD_ADDITIONAL,
                                out_ids: np.ndarray | None = None, out_dists: np.ndarray | None = None
                                ) -> CrossGroupStats:
        """ungx_build_cross_group_edges: ``vectors`` is a host array, or an integer device
        pointer with BUILD_VECTORS_ON_DEVICE in ``flags``."""
        st = CrossGroupStats()
        vp = vectors if (flags & BUILD_VECTORS_ON_DEVICE) else _ptr(vectors)
        io = None if intra_offsets is None else np.ascontiguousarray(intra_offsets, dtype=np.uint64)
        ic = None if intra_cols is None else np.ascontiguousarray(intra_cols, dtype=np.uint32)
        if ic is not None and ic.size == 0:
            ic = np.zeros(1, dtype=np.uint32)
        check(lib.ungx_build_cross_group_edges(self.h, vp, ctypes.byref(problem.c), _ptr(io), _ptr(ic), flags,
                                               _ptr(out_ids), _ptr(out_dists), ctypes.byref(st)), self.h)
        return st

    def graph_copy(self, num_points: int, num_cols: int) -> tuple[np.ndarray, np.ndarray]:
        """(offsets [n+1], cols) of the last ungx_build_cross_group_edges call."""
        off = np.empty(num_points + 1, dtype=np.uint64)
        cols = np.empty(max(num_cols, 1), dtype=np.uint32)
        check(lib.ungx_graph_copy(self.h, _ptr(off), _ptr(cols)))
        return off, cols[:num_cols]

    def exact_knn_graph_device(self, group_ranges: np.ndarray, cfg: ExactKnnConfig, d_graph: int,
                               d_entry_points: int | None = None, stream: int | None = None) -> float:
        """ungx_exact_knn_graph_device; group_ranges is [2 * groups] (first, end); returns kernel ms."""
        r = np.ascontiguousarray(group_ranges, dtype=np.uint32)
        ms = c_double(0.0)
        check(lib.ungx_exact_knn_graph_device(self.h, r.size // 2, _ptr(r) if r.size else None, ctypes.byref(cfg),
                                              d_graph, d_entry_points, stream, ctypes.byref(ms)), self.h)
        return ms.value

    def knn_rejected_rows(self) -> int:
        """Rows of the last tensor-route kNN seeding that the exact kernel rewrote."""
        return int(lib.ungx_exact_knn_rejected_rows(self.h))

    def knn_phase_ms(self) -> dict:
        """Device time of the last kNN seeding by phase (prefilter, rerank, fallback: the
        tensor route's; whole: the call; the gaps before the prefilter and the fallback)."""
        out = (c_double * 6)()
        lib.ungx_exact_knn_phase_ms(self.h, out)
        return {"prefilter": out[0], "rerank": out[1], "fallback": out[2], "whole": out[3],
                "before_prefilter": out[4], "before_fallback": out[5]}

    def graph_csr_device(self, num_points: int, topk: int, d_intra_offsets: int | None, d_intra_cols: int | None,
                         d_cross_ids: int | None, with_additional: bool, d_offsets: int, d_cols: int | None,
                         cols_capacity: int, stream: int | None = None) -> int:
        """ungx_graph_csr_device; returns the number of columns written."""
        total = c_uint64(0)
        check(lib.ungx_graph_csr_device(self.h, num_points, topk, d_intra_offsets, d_intra_cols, d_cross_ids,
                                        int(with_additional), d_offsets, d_cols, cols_capacity, ctypes.byref(total),
                                        stream), self.h)
        return int(total.value)


def exact_knn_default_config(candidate_k: int, final_degree: int) -> ExactKnnConfig:
    cfg = ExactKnnConfig()
    lib.ungx_exact_knn_default_config(candidate_k, final_degree, ctypes.byref(cfg))
    return cfg


def cross_edges_exact_noalloc(problem: Problem, d_vectors: int, d_ids: int, d_dists: int | None,
                              stream: int | None = None) -> None:
    """ungx_cross_edges_exact_noalloc: device pointers in and out, no device allocation."""
    check(lib.ungx_cross_edges_exact_noalloc(ctypes.byref(problem.c), d_vectors, d_ids, d_dists, stream))


def resident_bytes(num_points: int, dim: int, topk: int) -> int:
    """ungx_resident_bytes: device bytes of a resident build of this size."""
    return int(lib.ungx_resident_bytes(num_points, dim, topk))


def comm_id_create() -> bytes:
    """ungx_comm_id_create: a new NCCL unique id (128 bytes) for ungx_comm_init."""
    cid = CommId()
    check(lib.ungx_comm_id_create(ctypes.byref(cid)))
    return ctypes.string_at(ctypes.addressof(cid), ctypes.sizeof(cid))


def dist_slice(num_points: int, world_size: int, rank: int) -> tuple[int, int]:
    """(first row, row count) that ``rank`` passes from host memory to build_distributed."""
    a, c = c_uint32(), c_uint32()
    check(lib.ungx_dist_slice(num_points, world_size, rank, ctypes.byref(a), ctypes.byref(c)))
    return a.value, c.value


def graph_save_text(path: str, offsets: np.ndarray, cols: np.ndarray) -> None:
    """Write a CSR adjacency in the reference's graph text format (ungx_graph_save_text)."""
    offsets = np.ascontiguousarray(offsets, dtype=np.uint64)
    cols = np.ascontiguousarray(cols, dtype=np.uint32)
    check(lib.ungx_graph_save_text(os.fsencode(path), offsets.size - 1, _ptr(offsets), _ptr(cols)))


def flat_to_csr(flat_ids: np.ndarray, num_points: int, topk: int) -> tuple[np.ndarray, np.ndarray]:
    flat_ids = np.ascontiguousarray(flat_ids, dtype=np.uint32)
    off = np.empty(num_points + 1, dtype=np.uint64)
    check(lib.ungx_flat_to_csr(_ptr(flat_ids), num_points, topk, _ptr(off), None))
    cols = np.empty(max(int(off[-1]), 1), dtype=np.uint32)
    check(lib.ungx_flat_to_csr(_ptr(flat_ids), num_points, topk, _ptr(off), _ptr(cols)))
    return off, cols[:int(off[-1])]
