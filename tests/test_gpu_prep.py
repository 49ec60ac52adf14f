"""GPU parity of the device CSR canonicalisation (mfm_csr_prep_device) against
the oracle's restatement of the reference's `_prep_csr`
(python/modern_fm/_backend.py:44-52).

Integer work and duplicate sums in a fixed order: structure is compared
exactly, float64 values bitwise, float32 values bitwise against the oracle's
float64 result rounded once to float32.
"""

import numpy as np
import pytest

import golden_io
from oracle import oracle as O
from test_prep_csr import raw_csr

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _prep(ip, ix, dv, n_features, dtype):
    from modern_fm_b200.prep import prep_csr_device

    a, b, c = prep_csr_device(_dev(ip), _dev(ix), _dev(dv), n_features, dtype=dtype)
    torch.cuda.synchronize()
    return a.cpu().numpy(), b.cpu().numpy(), c.cpu().numpy()


def _check(ip, ix, dv, n_features):
    want = O.prep_csr(ip, ix, dv, n_features)
    for dtype in ("float64", "float32"):
        a, b, c = _prep(ip, ix, dv, n_features, dtype)
        assert np.array_equal(a, want[0])
        assert np.array_equal(b.astype(np.int64), want[1])
        ref = want[2] if dtype == "float64" else want[2].astype(np.float32)
        assert c.dtype == ref.dtype
        assert np.array_equal(c.view(np.uint8), ref.view(np.uint8)), dtype


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_short_rows_unsorted_with_duplicates(seed):
    rng = np.random.default_rng(seed)
    ip, ix, dv = raw_csr(rng, 3000, 200, [0, 1, 2, 7, 31, 32, 33, 39, 64, 255, 256], dup_pool=12)
    _check(ip, ix, dv, 200)


@pytest.mark.parametrize("n_features", [(1 << 24) - 1, 1 << 24, (1 << 24) + 1, 1 << 30])
def test_short_rows_at_the_sort_key_width_boundary(n_features):
    """Short rows are sorted on 32-bit keys (column << 8 | position) while
    every column fits in 24 bits and on 64-bit keys beyond; columns at the
    top of the range, duplicated, on both sides of the switch."""
    rng = np.random.default_rng(n_features % 1000)
    lens = [2, 39, 64, 65, 200, 256]
    top = np.arange(n_features - 40, n_features, dtype=np.int64)
    ip = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    ix = np.concatenate([rng.choice(top, size=n, replace=True) for n in lens]).astype(np.int64)
    dv = rng.normal(size=len(ix))
    _check(ip, ix, dv, n_features)


@pytest.mark.parametrize("seed", [0, 1])
def test_long_rows_unsorted_with_duplicates(seed):
    rng = np.random.default_rng(seed)
    lens = [257, 3, 300, 0, 1000, 39, 4095, 4096, 4097, 9000]
    ip, ix, dv = raw_csr(rng, 60, 5000, lens, dup_pool=40)
    _check(ip, ix, dv, 5000)
    ip, ix, dv = raw_csr(rng, 40, 1 << 22, lens)  # wide key space: all three sort passes
    _check(ip, ix, dv, 1 << 22)


def test_mixed_sorted_and_unsorted_rows():
    rng = np.random.default_rng(5)
    ip, ix, dv = raw_csr(rng, 500, 3000, [5, 39, 600], dup_pool=None, sort_rows=True)
    ix = ix.copy()
    lo, hi = ip[7], ip[8]
    ix[lo:hi] = ix[lo:hi][::-1].copy()  # one short row reversed
    lo, hi = ip[2], ip[3]
    ix[lo:hi] = ix[lo:hi][::-1].copy()  # one long row reversed
    _check(ip, ix, dv, 3000)


def test_canonical_input_passes_through():
    rng = np.random.default_rng(3)
    ip, ix, dv = raw_csr(rng, 2000, 1 << 16, [0, 13, 39, 300])
    keep = []
    for r in range(len(ip) - 1):  # make every row strictly increasing
        c = ix[ip[r]:ip[r + 1]]
        _, first = np.unique(c, return_index=True)
        keep.append(ip[r] + first[np.argsort(c[first], kind="stable")])
    sel = np.concatenate(keep)
    lens = np.array([len(k) for k in keep])
    ip2 = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    ix2, dv2 = ix[sel], dv[sel]
    a, b, c = _prep(ip2, ix2, dv2, 1 << 16, "float64")
    assert np.array_equal(a, ip2) and np.array_equal(b.astype(np.int64), ix2)
    assert np.array_equal(c.view(np.int64), dv2.view(np.int64))


def test_empty_shapes():
    _check(np.zeros(1, np.int64), np.zeros(0, np.int64), np.zeros(0), 4)
    _check(np.zeros(6, np.int64), np.zeros(0, np.int64), np.zeros(0), 4)


@pytest.mark.parametrize("bad", ["order", "range", "ends", "negative"])
def test_invalid_csr_raises_value_error(bad):
    ip = np.array([0, 2, 4], dtype=np.int64)
    ix = np.array([0, 1, 2, 3], dtype=np.int64)
    msg = "non-decreasing"
    if bad == "order":
        ip = np.array([0, 3, 2, 4], dtype=np.int64)
    elif bad == "range":
        ix = np.array([0, 1, 2, 9], dtype=np.int64)
        msg = "out of range"
    elif bad == "negative":
        ix = np.array([0, -1, 2, 3], dtype=np.int64)
        msg = "out of range"
    else:
        ip = np.array([0, 2, 3], dtype=np.int64)
        msg = "end at nnz"
    with pytest.raises(ValueError, match=msg):
        _prep(ip, ix, np.ones(4), 5, "float32")


def test_prepared_csr_scores_like_the_host_path():
    """Raw CSR -> device canonicalisation -> device FM scoring equals the
    oracle's FM scoring of the host-canonicalised CSR (float64, the reference's
    CUDA bar 1e-10)."""
    import ctypes as ct

    from modern_fm_b200 import _lib
    from modern_fm_b200.prep import prep_csr_device

    rng = np.random.default_rng(9)
    d, k = 400, 16
    ip, ix, dv = raw_csr(rng, 1500, d, [0, 4, 39, 80, 700], dup_pool=30)
    w0, w, V = 0.25, rng.normal(size=d), rng.normal(size=(d, k)) * 0.1
    a, b, c = prep_csr_device(_dev(ip), _dev(ix), _dev(dv), d, dtype="float64")
    n = len(ip) - 1
    out = torch.empty(n, dtype=torch.float64, device="cuda")
    wd, Vd = _dev(w), _dev(V)
    rc = _lib.lib().mfm_fm_predict_device(_lib.MFM_DTYPE_F64, 0, a.data_ptr(), b.data_ptr(),
                                          c.data_ptr(), n, ct.c_double(w0), wd.data_ptr(),
                                          Vd.data_ptr(), k, out.data_ptr(),
                                          torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    got = out.cpu().numpy()
    pp = O.prep_csr(ip, ix, dv, d)
    want = O.fm_predict_fast_csr(pp[0], pp[1], pp[2], d, w0, w, V)
    np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-10)


@pytest.mark.parametrize("case", golden_io.load("prep.npz"), ids=lambda c: c.name)
def test_device_prep_matches_reference_golden(case):
    """Against the reference's own `_prep_csr` output: structure exact; float64
    values bitwise where the duplicates' order is defined (`exact`), 1e-14
    otherwise; float32 values are those rounded once (one float32 ulp where
    the float64 sums differ in their last bit)."""
    ip, ix, dv, nf = case.a["indptr"], case.a["indices"], case.a["data"], case["n_features"]
    want = case.a["out_data"]
    for dtype in ("float64", "float32"):
        a, b, c = _prep(ip, ix, dv, nf, dtype)
        assert np.array_equal(a, case.a["out_indptr"])
        assert np.array_equal(b.astype(np.int64), case.a["out_indices"])
        ref = want if dtype == "float64" else want.astype(np.float32)
        if case["exact"]:
            assert np.array_equal(c.view(np.uint8), ref.view(np.uint8)), dtype
        elif dtype == "float64":
            np.testing.assert_allclose(c, ref, rtol=1e-14, atol=1e-14)
        else:
            np.testing.assert_allclose(c, ref, rtol=2.5e-7, atol=1e-12)
