"""GPU check of libffm loading onto the device (native reader, then
mfm_csr_prep_device) against fixtures made by the reference's own load_libffm:
float64 values bitwise, float32 values the reference's rounded once (NaN
entries compared as NaN)."""

import numpy as np
import pytest

import golden_io

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("case", [c for c in golden_io.load("libffm.npz") if c["error"] is None],
                         ids=lambda c: c.name)
def test_load_libffm_device_matches_reference_golden(tmp_path, case):
    from modern_fm_b200.libffm import load_libffm_device

    p = tmp_path / (case.name + ".ffm")
    p.write_bytes(case.a["text"].tobytes())
    for dtype in ("float64", "float32"):
        ip, ix, dv, y, f, nf = load_libffm_device(p, dtype=dtype)
        torch.cuda.synchronize()
        assert nf == case["n_features"]
        assert np.array_equal(ip.cpu().numpy(), case.a["indptr"])
        assert np.array_equal(ix.cpu().numpy().astype(np.int64), case.a["indices"])
        want = case.a["data"] if dtype == "float64" else case.a["data"].astype(np.float32)
        got = dv.cpu().numpy()
        assert got.dtype == want.dtype
        # NaN payloads may differ after a device float64 -> float32 conversion
        nan = np.isnan(want)
        assert np.array_equal(np.isnan(got), nan)
        assert np.array_equal(got[~nan].view(np.uint8), want[~nan].view(np.uint8))
        assert np.array_equal(y.cpu().numpy(), case.a["y"])
        assert np.array_equal(f, case.a["field_ids"])
