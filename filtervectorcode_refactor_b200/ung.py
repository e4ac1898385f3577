"""Host-side mirror of the reference's UniNavGraph build seam for the cross-edge path.

Method names, argument meaning and call order follow ``ANNS::UniNavGraph``
(UNG/codes/include/uni_nav_graph.h, UNG/codes/src/uni_nav_graph.cpp:54-146):

    build_trie_and_divide_groups      uni_nav_graph_label_graph.cpp:21-43
    prepare_group_storages_graphs     uni_nav_graph.cpp:148-181
    build_label_nav_graph             uni_nav_graph_label_graph.cpp:836-911
    build_cross_group_edges           uni_nav_graph_cross_edges.cpp:613-913
      build_cross_edges_generate_gpu_optimized   :334-440
      build_cross_edges_generate_additional      :442-596 (exact variant)
      add_offset_for_uni_nav_graph               uni_nav_graph.cpp:285-297
      merge_cross_edges_to_graph (+ additional)  :598-611

All computation runs in ``libungx.so`` (grouping and LNG on the host in C++, the
cross-edge top-k on the B200).  Error behaviour: the reference's GPU seam returns
``false`` on failure and ``build_cross_group_edges`` then falls back to a CPU path
unless ``UNG_CROSS_EDGE_GPU_STRICT=1`` (cross_edges.cpp:775-789).  This library has
no CPU path, so the seam returns ``False`` (with ``last_error`` set) and
``build_cross_group_edges`` raises, i.e. it behaves as the strict mode.
"""
from __future__ import annotations

import dataclasses

import numpy as np

from . import _native as nat

# CrossEdgeGpuWritebackMode, UNG/codes/include/ung_cross_edge_config.h:17-22
WRITEBACK_SEARCH_QUEUE = 0
WRITEBACK_ID_VECTOR = 1
WRITEBACK_FLAT_ID = 2


@dataclasses.dataclass
class CrossEdgeBuildTiming:
    """CrossEdgeBuildTiming, UNG/codes/include/ung_cross_edge_result.h:15-28 (fields this step owns)."""

    generate_ms: float = 0.0
    merge_cross_ms: float = 0.0
    output_storage_init_ms: float = 0.0
    gpu_h2d_ms: float = 0.0
    gpu_kernel_ms: float = 0.0
    gpu_d2h_ms: float = 0.0
    detail: dict = dataclasses.field(default_factory=dict)


class LabelNavGraph:
    """out_neighbors / in_neighbors as CSR over groups 1..G (index 0 unused)."""

    def __init__(self, out_offsets, out_ids, in_offsets, in_ids):
        self.out_offsets, self.out_ids = out_offsets, out_ids
        self.in_offsets, self.in_ids = in_offsets, in_ids

    def out_neighbors(self, g: int) -> np.ndarray:
        return self.out_ids[self.out_offsets[g]:self.out_offsets[g + 1]]

    def in_neighbors(self, g: int) -> np.ndarray:
        return self.in_ids[self.in_offsets[g]:self.in_offsets[g + 1]]


class UniNavGraph:
    def __init__(self, num_cross_edges: int = 6, device: int = 0, num_threads: int = 0,
                 route: int = nat.ROUTE_AUTO, shard_rank: int = 0, shard_count: int = 1):
        self._num_cross_edges = int(num_cross_edges)
        self._device = device
        self._num_threads = num_threads
        self._route = route
        self._shard_rank, self._shard_count = shard_rank, shard_count
        self._ctx: nat.Context | None = None
        self.last_error = ""
        self.timing = CrossEdgeBuildTiming()

    # ------------------------------------------------------------ input side
    def build_trie_and_divide_groups(self, label_offsets: np.ndarray, labels: np.ndarray) -> None:
        self._lg = nat.LabelGraph(label_offsets, labels, self._num_threads)
        self._num_points = self._lg.num_points
        self._num_groups = self._lg.num_groups
        self._group_id_to_range = self._lg.group_ranges.reshape(-1, 2)

    def prepare_group_storages_graphs(self, vectors: np.ndarray) -> None:
        """Reorder the base vectors so each group's rows are contiguous."""
        self._new_to_old_vec_ids = self._lg.new_to_old
        self._base = np.ascontiguousarray(vectors[self._new_to_old_vec_ids], dtype=np.float32)
        self._dim = self._base.shape[1]
        # groups 1..G hold consecutive row ranges that cover every row
        r = self._group_id_to_range.astype(np.int64)
        self._new_vec_id_to_group_id = np.repeat(np.arange(1, self._num_groups + 1, dtype=np.uint32),
                                                 r[1:, 1] - r[1:, 0])

    def build_label_nav_graph(self) -> None:
        self._label_nav_graph = LabelNavGraph(self._lg.out_offsets, self._lg.out_ids,
                                              self._lg.in_offsets, self._lg.in_ids)

    # ------------------------------------------------------------ cross edges
    def _problem(self) -> nat.Problem:
        return nat.Problem(self._num_points, self._dim, self._num_cross_edges, self._lg.group_ranges,
                           self._lg.out_offsets, self._lg.out_ids, None, self._route,
                           self._shard_rank, self._shard_count)

    def build_cross_edges_generate_gpu_optimized(self, writeback: int = WRITEBACK_FLAT_ID) -> bool:
        """Fills ``cross_group_neighbor_flat_ids`` ([n*k], UINT32_MAX = empty) and
        ``cross_group_neighbor_dists``; returns False on failure (message in last_error)."""
        try:
            if self._ctx is None:
                self._ctx = nat.Context(self._device)
            n, k = self._num_points, self._num_cross_edges
            self.cross_group_neighbor_flat_ids = np.full(n * k, nat.EMPTY_ID, dtype=np.uint32)
            self.cross_group_neighbor_dists = np.full(n * k, np.inf, dtype=np.float32)
            t = self._ctx.build(self._base, self._problem(), self.cross_group_neighbor_flat_ids,
                                self.cross_group_neighbor_dists)
        except nat.UngxError as e:
            self.last_error = str(e)
            return False
        d = t.as_dict()
        self.timing.generate_ms += d["generate_ms"]
        self.timing.gpu_h2d_ms += d["gpu_h2d_ms"]
        self.timing.gpu_kernel_ms += d["gpu_kernel_ms"]
        self.timing.gpu_d2h_ms += d["gpu_d2h_ms"]
        self.timing.detail = d
        self._writeback = writeback
        return True

    def search_queue(self, point: int) -> list[tuple[int, float]]:
        """The (id, distance) content of the reference's SearchQueue of ``point``."""
        k = self._num_cross_edges
        ids = self.cross_group_neighbor_flat_ids[point * k:(point + 1) * k]
        ds = self.cross_group_neighbor_dists[point * k:(point + 1) * k]
        return [(int(i), float(x)) for i, x in zip(ids, ds) if i != nat.EMPTY_ID]

    def build_cross_group_edges(self, intra_offsets: np.ndarray | None = None, intra_cols: np.ndarray | None = None,
                                intra_ids_are_global: bool = False, additional_edges: bool = True) -> None:
        """UniNavGraph::build_cross_group_edges (uni_nav_graph_cross_edges.cpp:613-913) in one
        library call (ungx_build_cross_group_edges): the GPU cross edges, the exact
        additional edges, add_offset_for_uni_nav_graph on the intra-group graph (CSR over
        reordered points, group-local ids unless ``intra_ids_are_global``) and the merge.
        Fills ``cross_group_neighbor_flat_ids`` / ``_dists`` and the merged adjacency
        ``graph_offsets`` / ``graph_cols`` (per point: intra edges, cross edges nearest
        first, additional edges).  Raises on failure: the library has no CPU path, so
        this is the reference's strict mode."""
        try:
            if self._ctx is None:
                self._ctx = nat.Context(self._device)
            n, k = self._num_points, self._num_cross_edges
            self.cross_group_neighbor_flat_ids = np.full(n * k, nat.EMPTY_ID, dtype=np.uint32)
            self.cross_group_neighbor_dists = np.full(n * k, np.inf, dtype=np.float32)
            flags = nat.BUILD_ADDITIONAL if additional_edges else 0
            if intra_offsets is not None and not intra_ids_are_global:
                flags |= nat.BUILD_INTRA_LOCAL_IDS
            st = self._ctx.build_cross_group_edges(self._base, self._problem(), intra_offsets, intra_cols, flags,
                                                   self.cross_group_neighbor_flat_ids,
                                                   self.cross_group_neighbor_dists)
            self.graph_offsets, self.graph_cols = self._ctx.graph_copy(n, int(st.num_cols))
        except nat.UngxError as e:
            self.last_error = str(e)
            raise RuntimeError("GPU cross-group edge build failed (no CPU path in this library): " + str(e)) from e
        d = st.cross.as_dict()
        self.timing.generate_ms += d["generate_ms"]
        self.timing.gpu_h2d_ms += d["gpu_h2d_ms"]
        self.timing.gpu_kernel_ms += d["gpu_kernel_ms"]
        self.timing.gpu_d2h_ms += d["gpu_d2h_ms"]
        self.timing.merge_cross_ms += st.merge_ms
        self.timing.detail = dict(d, additional=st.additional.as_dict(), cross_edges=int(st.cross_edges),
                                  num_cols=int(st.num_cols), total_ms=st.total_ms)
        self.additional_edge_count = int(st.additional.edges)

    def cross_edges_csr(self) -> tuple[np.ndarray, np.ndarray]:
        """CrossEdgeGraphMaterializationWriter::build_csr_adjacency
        (UNG/codes/src/ung_cross_edge_output_writer.cpp:44-66)."""
        return nat.flat_to_csr(self.cross_group_neighbor_flat_ids, self._num_points, self._num_cross_edges)

    def build(self, vectors: np.ndarray, label_offsets: np.ndarray, labels: np.ndarray) -> None:
        """The cross-edge slice of UniNavGraph::build (uni_nav_graph.cpp:54-146)."""
        self.build_trie_and_divide_groups(label_offsets, labels)
        self.prepare_group_storages_graphs(vectors)
        self.build_label_nav_graph()
        self.build_cross_group_edges()

    def close(self) -> None:
        if self._ctx is not None:
            self._ctx.close()
            self._ctx = None
