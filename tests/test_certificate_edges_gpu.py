"""The tensor-core route's rounding certificate on inputs built to break it
(tests/adversarial.py): rows whose norms span six decades in one group pair, operand
elements below or around fp16's smallest normal value after the power-of-two scale,
an element no fp16 scale can hold (every row rescanned exactly), a large common
offset, and coarse values with ties.  Whatever the certificate decides, the rows
must equal the reference's exact scan in ids and distance bits; the exact route is
checked on the same inputs."""
import numpy as np
import pytest

import oracle as O
from adversarial import CASES, make_case
from filtervectorcode_refactor_b200 import _native as nat
from parity import assert_rows_match

pytestmark = pytest.mark.gpu


def expected(case):
    X, k, first, ranges, off, ids = case
    ref = O.reference()
    impl = ref if ref is not None else O.oracle()
    e_ids, e_d, _ = impl.cross_exact(X, k, first, off, ids)
    return e_ids, e_d


@pytest.fixture(scope="module")
def ctx():
    c = nat.Context(0)
    yield c
    c.close()


@pytest.mark.parametrize("route", [nat.ROUTE_TENSOR, nat.ROUTE_EXACT], ids=["tensor", "exact"])
@pytest.mark.parametrize("name", CASES)
def test_certificate_edge_case(ctx, name, route):
    case = make_case(name)
    X, k, first, ranges, off, ids = case
    n, d = X.shape
    e_ids, e_d = expected(case)
    prob = nat.Problem(n, d, k, ranges, off, ids, route=route)
    got_ids = np.full(n * k, 3, dtype=np.uint32)
    got_d = np.full(n * k, -2, dtype=np.float32)
    ctx.prepare_base_vectors(X, n, d, on_device=False)
    try:
        t = ctx.generate(prob, got_ids, got_d)
    finally:
        ctx.release_base_vectors()
    assert_rows_match(got_ids, got_d, e_ids, e_d, k)
    if route == nat.ROUTE_TENSOR:
        rows = t.rows_certified + t.rows_fallback
        assert rows == int(np.diff(ranges.reshape(-1, 2)[[1, 2, 4]], axis=1).sum())  # rows of groups 1, 2, 4
        if name == "exact_only":
            assert t.rows_certified == 0 and t.rows_fallback == rows
        print(f"{name}: certified {t.rows_certified} rescanned {t.rows_fallback}")


@pytest.mark.parametrize("outlier_row", [None, 1000, 1001], ids=["none", "sampled", "unsampled"])
def test_sampled_operand_scale(ctx, outlier_row):
    """Above 2^18 rows the operand's mean and scale come from a row sample (every 4th row
    here). An element far beyond the sample's range, in a row the sample skips, overflows
    the sampled scale: the gated full pass must redo the operand, and the rows stay equal
    to the exact scan. The same element in a sampled row, and no outlier at all, take the
    sampled scale as it is."""
    from adversarial import _groups
    rng = np.random.default_rng(5)
    sizes = [1000, 3000, 296000]
    first, ranges, off, ids = _groups(sizes, {1: [2]})
    n, d, k = sum(sizes), 16, 6
    X = rng.standard_normal((n, d)).astype(np.float32)
    if outlier_row is not None:
        X[outlier_row, 3] = np.float32(1.0e3)
    e_ids, e_d, _ = O.oracle().cross_exact(X, k, first, off, ids)
    prob = nat.Problem(n, d, k, ranges, off, ids, route=nat.ROUTE_TENSOR)
    got_ids = np.full(n * k, 3, dtype=np.uint32)
    got_d = np.full(n * k, -2, dtype=np.float32)
    ctx.prepare_base_vectors(X, n, d, on_device=False)
    try:
        t = ctx.generate(prob, got_ids, got_d)
    finally:
        ctx.release_base_vectors()
    assert_rows_match(got_ids, got_d, e_ids, e_d, k)
    print(f"outlier {outlier_row}: certified {t.rows_certified} rescanned {t.rows_fallback}")
