"""Seeded synthetic CTR workloads with the shapes of the benchmark configurations.

No dataset or network access is assumed: each generator draws its CSR matrix,
labels and (where the configuration plants them) ground-truth parameters from
a numpy Generator seeded by `seed`, so every run sees identical inputs. CSR
arrays are in the reference's boundary format (int64 indptr/indices, float64
data, canonical: sorted, duplicate-free rows).

  onehot_ctr  16 one-hot fields x 16 categories (256 features, 16 nnz/row),
              labels from 8 planted field-pair tables (FM / FFM workloads).
  ctr_fm      39 fields: 13 numeric (one reserved id each, log1p(LogNormal(0,2)))
              + 26 categorical (per-field Zipf(1.1) over 2^20, hashed into 2^22),
              labels from a planted FM at ~3 % positives.
  fwfm_ctr    9 one-hot fields, Zipf(1.05) ids, ~373k features, planted FwFM,
              4.4 % positives.
  softmax_ctr ragged rows (Poisson(30)+1 nnz), uniform ids over 1M features,
              LogNormal(0,1) values, 10 classes from a planted FM + Gumbel noise.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import scipy.sparse as sp

_MASK = np.uint64(0xFFFFFFFFFFFFFFFF)


@dataclass
class Csr:
    indptr: np.ndarray
    indices: np.ndarray
    data: np.ndarray
    n_features: int

    @property
    def n_rows(self):
        return len(self.indptr) - 1

    @property
    def nnz(self):
        return len(self.data)

    def scipy(self):
        return sp.csr_matrix((self.data, self.indices, self.indptr),
                             shape=(self.n_rows, self.n_features))

    def rows(self, lo, hi):
        a, b = self.indptr[lo], self.indptr[hi]
        return Csr(self.indptr[lo:hi + 1] - a, self.indices[a:b], self.data[a:b],
                   self.n_features)


def splitmix64(x: np.ndarray) -> np.ndarray:
    """SplitMix64 finaliser (Steele, Lea, Flood 2014) on uint64 arrays."""
    with np.errstate(over="ignore"):
        z = (x.astype(np.uint64) + np.uint64(0x9E3779B97F4A7C15)) & _MASK
        z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & _MASK
        z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & _MASK
        return z ^ (z >> np.uint64(31))


def zipf_ids(rng, s, vocab, size, head=4096):
    """Bounded Zipf(s) ranks in [0, vocab) (rank r has mass ~ (r+1)^-s).

    Inverse CDF: exact over the `head` most frequent ranks (a cache-resident
    table searched through a 2^16-bucket guide table), and for the tail the
    inverse of the continuous power law carrying the same remaining mass
    (rank r covers [r + 1/2, r + 3/2))."""
    head = min(head, vocab)
    w = np.arange(1, head + 1, dtype=np.float64) ** (-s)
    a = 1.0 - s
    lo, hi = head + 0.5, vocab + 0.5  # continuous tail on [lo, hi)
    tail = (hi ** a - lo ** a) / a if vocab > head else 0.0
    total = w.sum() + tail
    cdf = np.cumsum(w) / total
    u = rng.random(size)
    nb = 1 << 16
    guide = np.searchsorted(cdf, np.arange(nb, dtype=np.float64) / nb, side="right")
    out = guide[np.minimum((u * nb).astype(np.int64), nb - 1)].astype(np.int64)
    cdf_pad = np.append(cdf, 2.0)
    while True:  # advance to the first rank whose cdf exceeds u (a few steps)
        step = (out < head) & (cdf_pad[np.minimum(out, head)] <= u)
        if not step.any():
            break
        out += step
    t = out >= head
    if t.any():
        ut = (u[t] - cdf[-1]) * total  # mass into the tail
        x = np.exp(np.log(lo ** a + a * ut) / a)
        out[t] = np.clip(np.floor(x - 0.5).astype(np.int64), head, vocab - 1)
    return out


def _canonical(rows_idx, rows_val, n_features):
    """(n, z) index/value blocks -> canonical CSR (sorted, duplicates summed)."""
    n, z = rows_idx.shape
    order = np.argsort(rows_idx, axis=1, kind="stable")
    idx = np.take_along_axis(rows_idx, order, 1)
    val = np.take_along_axis(rows_val, order, 1).astype(np.float64)
    dup = np.zeros((n, z), dtype=bool)
    dup[:, 1:] = idx[:, 1:] == idx[:, :-1]
    for r, j in zip(*np.nonzero(dup)):  # rare hash collisions: fold into the first copy
        j0 = j - 1
        while dup[r, j0]:
            j0 -= 1
        val[r, j0] += val[r, j]
    keep = ~dup
    counts = keep.sum(axis=1)
    indptr = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    return Csr(indptr, idx[keep].astype(np.int64), val[keep], n_features)


def _fm_scores(X: Csr, w0, w, V):
    M = X.scipy()
    xv = M @ V
    x2v2 = M.multiply(M) @ (V * V)
    return w0 + M @ w + 0.5 * (xv * xv - x2v2).sum(axis=1)


def _bias_for_rate(scores, rate):
    """b such that mean(sigmoid(scores + b)) == rate (bisection)."""
    lo, hi = -50.0, 50.0
    for _ in range(80):
        mid = 0.5 * (lo + hi)
        if np.mean(1.0 / (1.0 + np.exp(-(scores + mid)))) > rate:
            hi = mid
        else:
            lo = mid
    return 0.5 * (lo + hi)


def onehot_ctr(n_rows, seed, n_fields=16, n_cats=16, n_pairs=8):
    """Planted-interaction CTR: one uniform category per field (feature
    n_cats*f + c, value 1.0); y ~ Bernoulli(sigmoid(-0.5 + sum of 8 field-pair
    N(0, 1.5) table entries + N(0, 0.3) per-feature linear terms)).
    Returns (Csr, y, field_ids)."""
    rng = np.random.default_rng(seed)
    d = n_fields * n_cats
    cats = rng.integers(0, n_cats, size=(n_rows, n_fields))
    idx = cats + n_cats * np.arange(n_fields)[None, :]
    X = Csr(np.arange(0, n_rows * n_fields + 1, n_fields, dtype=np.int64),
            idx.ravel().astype(np.int64), np.ones(n_rows * n_fields), d)
    pairs = set()
    while len(pairs) < n_pairs:
        a, b = sorted(rng.choice(n_fields, size=2, replace=False))
        pairs.add((int(a), int(b)))
    s = np.full(n_rows, -0.5)
    for a, b in sorted(pairs):
        table = rng.normal(0.0, 1.5, size=(n_cats, n_cats))
        s += table[cats[:, a], cats[:, b]]
    lin = rng.normal(0.0, 0.3, size=d)
    s += lin[idx].sum(axis=1)
    y = (rng.random(n_rows) < 1.0 / (1.0 + np.exp(-s))).astype(np.float64)
    field_ids = np.arange(d, dtype=np.int64) // n_cats
    return X, y, field_ids


def ctr_fm(n_rows, seed, n_numeric=13, n_cat=26, vocab=2**20, space=2**22, zipf_s=1.1,
           k=16, labels=False, positive_rate=0.03):
    """Large CTR-shaped FM input. Returns (Csr, y or None)."""
    rng = np.random.default_rng(seed)
    num_val = np.log1p(np.exp(rng.normal(0.0, 2.0, size=(n_rows, n_numeric))))
    ranks = zipf_ids(rng, zipf_s, vocab, (n_rows, n_cat))
    key = (np.arange(n_cat, dtype=np.uint64)[None, :] * np.uint64(vocab)
           + ranks.astype(np.uint64))
    cat_idx = (splitmix64(key) % np.uint64(space - n_numeric)).astype(np.int64) + n_numeric
    idx = np.concatenate([np.broadcast_to(np.arange(n_numeric), (n_rows, n_numeric)),
                          cat_idx], axis=1)
    val = np.concatenate([num_val, np.ones((n_rows, n_cat))], axis=1)
    X = _canonical(idx, val, space)
    y = None
    if labels:
        prng = np.random.default_rng(seed + 1_000_003)
        w = prng.normal(0.0, 0.1, size=space)
        V = prng.normal(0.0, 0.1, size=(space, k))
        s = _fm_scores(X, 0.0, w, V)
        s = s + _bias_for_rate(s, positive_rate)
        y = (rng.random(n_rows) < 1.0 / (1.0 + np.exp(-s))).astype(np.float64)
    return X, y


FWFM_VOCABS = (100_000, 80_000, 60_000, 50_000, 40_000, 25_000, 10_000, 5_000, 3_000)


def fwfm_ctr(n_rows, seed, vocabs=FWFM_VOCABS, zipf_s=1.05, k=8, positive_rate=0.044,
             labels=True):
    """One-hot FwFM workload. Returns (Csr, y, field_ids); y is None when
    `labels` is false (the planted-model scoring is skipped)."""
    rng = np.random.default_rng(seed)
    F = len(vocabs)
    offs = np.concatenate([[0], np.cumsum(vocabs)]).astype(np.int64)
    d = int(offs[-1])
    idx = np.stack([zipf_ids(rng, zipf_s, v, n_rows) + offs[f] for f, v in enumerate(vocabs)],
                   axis=1)
    X = Csr(np.arange(0, n_rows * F + 1, F, dtype=np.int64), idx.ravel().astype(np.int64),
            np.ones(n_rows * F), d)
    field_ids = np.repeat(np.arange(F, dtype=np.int64), vocabs)
    if not labels:
        return X, None, field_ids
    prng = np.random.default_rng(seed + 1_000_003)
    r = prng.uniform(0.0, 1.0, size=(F, F))
    V = prng.normal(0.0, 0.2, size=(d, k))
    Vi = V[idx]  # (n, F, k)
    s = np.zeros(n_rows)
    for a in range(F):
        for b in range(a + 1, F):
            s += r[a, b] * np.einsum("nk,nk->n", Vi[:, a], Vi[:, b])
    s = s + _bias_for_rate(s, positive_rate)
    y = (rng.random(n_rows) < 1.0 / (1.0 + np.exp(-s))).astype(np.float64)
    return X, y, field_ids


def softmax_ctr(n_rows, seed, n_features=1_000_000, n_classes=10, mean_nnz=30, k=8,
                score_fn=None):
    """Ragged multiclass workload. Returns (Csr, y (int64), sample_weight).
    `score_fn(X, w0, w, V)` scores the planted per-class FMs (default: scipy
    on the host; a GPU scorer gives the same labels up to rounding, faster)."""
    rng = np.random.default_rng(seed)
    z = rng.poisson(mean_nnz, size=n_rows) + 1
    indptr = np.concatenate([[0], np.cumsum(z)]).astype(np.int64)
    ids = rng.integers(0, n_features, size=int(indptr[-1]))
    vals = rng.lognormal(0.0, 1.0, size=int(indptr[-1]))
    M = sp.csr_matrix((vals, ids, indptr), shape=(n_rows, n_features))
    M.sum_duplicates()
    X = Csr(M.indptr.astype(np.int64), M.indices.astype(np.int64), M.data.astype(np.float64),
            n_features)
    prng = np.random.default_rng(seed + 1_000_003)
    logits = np.empty((n_rows, n_classes))
    for c in range(n_classes):
        w = prng.normal(0.0, 0.1, size=n_features)
        V = prng.normal(0.0, 0.1, size=(n_features, k))
        logits[:, c] = (score_fn or _fm_scores)(X, 0.0, w, V)
    logits += rng.gumbel(size=logits.shape)
    y = logits.argmax(axis=1).astype(np.int64)
    sw = rng.uniform(0.5, 2.0, size=n_rows)
    return X, y, sw


def row_orders(n_rows, epochs, seed):
    """(epochs, n_rows) visit order, one permutation per epoch."""
    rng = np.random.default_rng(seed)
    return np.stack([rng.permutation(n_rows) for _ in range(epochs)]).astype(np.int64)


# ---------------------------------------------------------------------------
# device-side generator for the large CTR workload (torch is used as plumbing
# only: random numbers, sorting and buffers on the GPU)
# ---------------------------------------------------------------------------


def _mix32(t):
    """32-bit avalanche (MurmurHash3 fmix32) on an int64 tensor holding
    non-negative 32-bit values."""
    m = 0xFFFFFFFF
    t = t & m
    t = ((t ^ (t >> 16)) * 0x85EBCA6B) & m
    t = ((t ^ (t >> 13)) * 0xC2B2AE35) & m
    return t ^ (t >> 16)


def ctr_fm_torch(n_rows, seed, device="cuda", n_numeric=13, n_cat=26, vocab=2**20,
                 space=2**22, zipf_s=1.1, head=4096, value_dtype=None):
    """The ctr_fm workload drawn on the GPU (same distributions as `ctr_fm`,
    different random stream). Returns a dict of device tensors:
    indptr int64 (n+1), indices int32 (nnz), data (nnz) in `value_dtype`
    (default float32; the values are drawn in float64), n_features.
    Rows are canonical: sorted, duplicate-free (a rare in-row hash collision
    is moved to the next free id)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    n = int(n_rows)
    num_val = torch.log1p(torch.exp(torch.randn(n, n_numeric, generator=g, device=device,
                                                dtype=torch.float64) * 2.0))
    # bounded Zipf ranks: exact head table + continuous power-law tail
    w = torch.arange(1, head + 1, dtype=torch.float64, device=device) ** (-zipf_s)
    a = 1.0 - zipf_s
    lo, hi = head + 0.5, vocab + 0.5
    tail = (hi ** a - lo ** a) / a
    total = float(w.sum()) + tail
    cdf = torch.cumsum(w, 0) / total
    u = torch.rand(n, n_cat, generator=g, device=device, dtype=torch.float64)
    ranks = torch.searchsorted(cdf, u, right=True)
    t = ranks >= head
    x = torch.exp(torch.log(lo ** a + a * (u - cdf[-1]) * total) / a)
    tail_r = torch.clamp(torch.floor(x - 0.5), head, vocab - 1).to(torch.int64)
    ranks = torch.where(t, tail_r, ranks)
    field = torch.arange(n_cat, device=device, dtype=torch.int64)[None, :]
    h = _mix32(_mix32(ranks * 0x9E3779B1 + field * 0x7FEB352D) + field)
    ids = h % (space - n_numeric) + n_numeric
    for _ in range(8):  # resolve rare in-row collisions deterministically
        ids, _ = torch.sort(ids, dim=1)
        dup = torch.zeros_like(ids, dtype=torch.bool)
        dup[:, 1:] = ids[:, 1:] == ids[:, :-1]
        if not bool(dup.any()):
            break
        ids = torch.where(dup, (ids - n_numeric + 1) % (space - n_numeric) + n_numeric, ids)
    idx = torch.cat([torch.arange(n_numeric, device=device).expand(n, n_numeric), ids], 1)
    val = torch.cat([num_val, torch.ones(n, n_cat, device=device, dtype=torch.float64)], 1)
    z = n_numeric + n_cat
    indptr = torch.arange(0, n * z + 1, z, device=device, dtype=torch.int64)
    return dict(indptr=indptr, indices=idx.reshape(-1).to(torch.int32).contiguous(),
                data=val.reshape(-1).to(value_dtype or torch.float32).contiguous(),
                n_features=space)
