"""CPU checks of the CSR canonicalisation step.

The oracle's `prep_csr` restates the reference's `_prep_csr`
(python/modern_fm/_backend.py:44-52: `X.tocsr().astype(np.float64);
X.sum_duplicates()`). It is pinned here against scipy, which is that step's
implementation: identical structure always, identical values wherever scipy
adds a column's duplicates in their original order (rows scipy does not
reorder, at most two duplicates of a column), 1e-14 relative otherwise.
"""

import numpy as np
import pytest
import scipy.sparse as sp

import golden_io
from oracle import oracle as O


def raw_csr(rng, n_rows, n_features, lens, dup_pool=None, sort_rows=False):
    """A CSR with rows of the given lengths, columns drawn with repeats from
    `dup_pool` columns per row (None: any column), values N(0, 1) with some
    explicit zeros and negative zeros."""
    ip, ix, dv = [0], [], []
    for r in range(n_rows):
        L = int(lens[r % len(lens)])
        if dup_pool is None:
            c = rng.integers(0, n_features, size=L)
        else:
            pool = min(dup_pool, n_features)
            base = rng.choice(n_features, size=pool, replace=False)
            c = base[rng.integers(0, pool, size=L)]
        if sort_rows:
            c = np.sort(c, kind="stable")
        v = rng.normal(size=L)
        v[rng.random(L) < 0.05] = 0.0
        v[rng.random(L) < 0.02] = -0.0
        ix.extend(c.tolist())
        dv.extend(v.tolist())
        ip.append(len(ix))
    return (np.array(ip, dtype=np.int64), np.array(ix, dtype=np.int64),
            np.array(dv, dtype=np.float64))


def scipy_prep(ip, ix, dv, n_features):
    """The reference's _prep_csr on the same arrays."""
    X = sp.csr_matrix((dv.copy(), ix.copy(), ip.copy()), shape=(len(ip) - 1, n_features))
    X = X.tocsr().astype(np.float64)
    X.sum_duplicates()
    return X.indptr.astype(np.int64), X.indices.astype(np.int64), X.data


def max_dups_per_column(ip, ix):
    m = 0
    for r in range(len(ip) - 1):
        _, c = np.unique(ix[ip[r]:ip[r + 1]], return_counts=True)
        if len(c):
            m = max(m, int(c.max()))
    return m


def test_canonical_input_is_unchanged():
    rng = np.random.default_rng(0)
    X = sp.random(300, 500, density=0.05, format="csr", random_state=1)
    ip, ix, dv = X.indptr.astype(np.int64), X.indices.astype(np.int64), X.data
    a, b, c = O.prep_csr(ip, ix, dv, 500)
    assert np.array_equal(a, ip) and np.array_equal(b, ix)
    assert np.array_equal(c.view(np.int64), dv.view(np.int64))
    del rng


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_sorted_rows_with_duplicates_bitwise(seed):
    rng = np.random.default_rng(seed)
    ip, ix, dv = raw_csr(rng, 200, 64, [0, 1, 5, 39, 300], dup_pool=8, sort_rows=True)
    want = scipy_prep(ip, ix, dv, 64)
    got = O.prep_csr(ip, ix, dv, 64)
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1])
    assert np.array_equal(got[2].view(np.int64), want[2].view(np.int64))


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_unsorted_rows_at_most_two_duplicates_bitwise(seed):
    rng = np.random.default_rng(seed)
    ip, ix, dv = raw_csr(rng, 300, 1 << 20, [3, 17, 39, 400])
    assert max_dups_per_column(ip, ix) <= 2
    want = scipy_prep(ip, ix, dv, 1 << 20)
    got = O.prep_csr(ip, ix, dv, 1 << 20)
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1])
    assert np.array_equal(got[2].view(np.int64), want[2].view(np.int64))


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_unsorted_rows_many_duplicates(seed):
    rng = np.random.default_rng(seed)
    ip, ix, dv = raw_csr(rng, 300, 50, [0, 2, 31, 64, 257, 1000], dup_pool=6)
    want = scipy_prep(ip, ix, dv, 50)
    got = O.prep_csr(ip, ix, dv, 50)
    assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1])
    np.testing.assert_allclose(got[2], want[2], rtol=1e-14, atol=1e-14)


def test_explicit_zeros_and_empty():
    ip = np.array([0, 0, 3, 3, 5], dtype=np.int64)
    ix = np.array([4, 1, 4, 2, 2], dtype=np.int64)
    dv = np.array([1.5, 0.0, -1.5, -0.0, -0.0])
    a, b, c = O.prep_csr(ip, ix, dv, 6)
    assert a.tolist() == [0, 0, 2, 2, 3]
    assert b.tolist() == [1, 4, 2]
    assert c.tolist() == [0.0, 0.0, 0.0]
    assert np.signbit(c[2])  # -0.0 + -0.0 keeps its sign, as in scipy
    a, b, c = O.prep_csr(np.zeros(1, dtype=np.int64), np.zeros(0, np.int64), np.zeros(0), 3)
    assert a.tolist() == [0] and len(b) == 0 and len(c) == 0


@pytest.mark.parametrize("bad", ["order", "range", "ends"])
def test_invalid_csr_raises(bad):
    ip = np.array([0, 2, 4], dtype=np.int64)
    ix = np.array([0, 1, 2, 3], dtype=np.int64)
    if bad == "order":
        ip = np.array([0, 3, 2, 4], dtype=np.int64)
    elif bad == "range":
        ix = np.array([0, 1, 2, 9], dtype=np.int64)
    else:
        ip = np.array([0, 2, 3], dtype=np.int64)
    with pytest.raises(ValueError):
        O.prep_csr(ip, ix, np.ones(4), 5)


def test_device_wrapper_rejects_host_tensors():
    torch = pytest.importorskip("torch")
    from modern_fm_b200.prep import prep_csr_device

    with pytest.raises(ValueError):
        prep_csr_device(torch.zeros(2, dtype=torch.int64), torch.zeros(1, dtype=torch.int64),
                        torch.zeros(1, dtype=torch.float64), 4)


@pytest.mark.parametrize("case", golden_io.load("prep.npz"), ids=lambda c: c.name)
def test_oracle_matches_reference_prep_golden(case):
    """Fixtures from the reference's own `_prep_csr` (tests/golden/make_golden.py)."""
    got = O.prep_csr(case.a["indptr"], case.a["indices"], case.a["data"], case["n_features"])
    assert np.array_equal(got[0], case.a["out_indptr"])
    assert np.array_equal(got[1], case.a["out_indices"])
    if case["exact"]:
        assert np.array_equal(got[2].view(np.int64), case.a["out_data"].view(np.int64))
    else:
        np.testing.assert_allclose(got[2], case.a["out_data"], rtol=1e-14, atol=1e-14)
