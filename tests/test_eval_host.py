"""CPU checks of the validation-metric restatement used to check the device
early-stopping evaluation (mfm_fm_eval_device), pinned by known answers of
the reference's losses (python/modern_fm/losses.py:25-68)."""

import math

import numpy as np
import pytest

import golden_io
from oracle import oracle as O


def test_logistic_loss_known_answers():
    # s = 0: log 2 whatever the label
    assert O.logistic_loss([0.0, 1.0], [0.0, 0.0]) == pytest.approx(math.log(2.0), rel=1e-15)
    # large |s|: the loss is the margin on the wrong side, ~0 on the right one
    assert O.logistic_loss([0.0], [40.0]) == pytest.approx(40.0, rel=1e-15)
    assert O.logistic_loss([1.0], [40.0]) == pytest.approx(math.exp(-40.0), rel=1e-12)
    # label smoothing eps moves the target to y (1 - eps) + eps / 2
    s, eps = 1.3, 0.1
    t = 1.0 * (1 - eps) + 0.5 * eps
    want = max(s, 0.0) - s * t + math.log1p(math.exp(-abs(s)))
    assert O.logistic_loss([1.0], [s], label_smoothing=eps) == pytest.approx(want, rel=1e-15)


def test_squared_loss_and_weights():
    assert O.squared_loss([1.0, 3.0], [2.0, 1.0]) == pytest.approx((0.5 + 2.0) / 2, rel=1e-15)
    got = O.squared_loss([1.0, 3.0], [2.0, 1.0], sample_weight=[1.0, 3.0])
    assert got == pytest.approx((0.5 * 1 + 2.0 * 3) / 4.0, rel=1e-15)
    assert np.isnan(O.squared_loss(np.zeros(0), np.zeros(0)))


def test_device_eval_rejects_host_tensors():
    torch = pytest.importorskip("torch")
    from modern_fm_b200.evaluate import fm_eval_device

    z64 = torch.zeros(2, dtype=torch.int64)
    with pytest.raises(ValueError):
        fm_eval_device(z64, torch.zeros(1, dtype=torch.int32), torch.zeros(1), 0.0,
                       torch.zeros(3), torch.zeros(3, 2), torch.zeros(1, dtype=torch.float64))


@pytest.mark.parametrize("case", golden_io.load("losses.npz"), ids=lambda c: c.name)
def test_oracle_losses_match_reference_golden(case):
    """Fixtures from the reference's own losses.py (tests/golden/make_golden.py):
    the same NumPy expressions, so the values are equal bitwise."""
    sw = case.a["sample_weight"] if case["weighted"] else None
    if case["loss"] == "logistic":
        got = O.logistic_loss(case.a["y"], case.a["raw"], label_smoothing=case["label_smoothing"],
                              sample_weight=sw)
    else:
        got = O.squared_loss(case.a["y"], case.a["raw"], sample_weight=sw)
    assert got == case.a["value"][0]
