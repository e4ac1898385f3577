"""B200-native UNG cross-group edge builder (drop-in for the cross-edge step of
panjd123/FilterVectorCode_refactor's UniNavGraph build).

The compute lives in ``libungx.so`` (C ABI, include/ungx.h); this package is its
host-side mirror of the reference interface plus seeded input generators.
"""
from . import _native
from ._native import (EMPTY_ID, ROUTE_AUTO, ROUTE_EXACT, ROUTE_TENSOR, Context, CrossEdgeTiming, LabelGraph,
                      Problem, UngxError)
from .ung import UniNavGraph

__all__ = ["EMPTY_ID", "ROUTE_AUTO", "ROUTE_EXACT", "ROUTE_TENSOR", "Context", "CrossEdgeTiming", "LabelGraph",
           "Problem", "UngxError", "UniNavGraph", "_native"]
