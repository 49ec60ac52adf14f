"""Loader for the fixtures in tests/golden/ (made by tests/golden/make_golden.py)."""

import json
import os

import numpy as np
import scipy.sparse as sp

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


class Case(dict):
    """Case metadata (dict) plus its arrays as attributes via `a[...]`."""

    def __init__(self, meta, arrays):
        super().__init__(meta)
        self.a = arrays

    @property
    def name(self):
        return self["name"]

    def dense(self):
        n_rows = len(self.a["indptr"]) - 1
        X = sp.csr_matrix((self.a["data"], self.a["indices"], self.a["indptr"]),
                          shape=(n_rows, self["n_features"]))
        return X.toarray()


def load(fname):
    z = np.load(os.path.join(GOLDEN, fname))
    metas = json.loads(bytes(z["__cases__"]).decode())
    out = []
    for m in metas:
        pre = m["name"] + "/"
        arrays = {k[len(pre):]: z[k] for k in z.files if k.startswith(pre)}
        out.append(Case(m, arrays))
    return out
