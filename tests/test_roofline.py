"""The performance model (se12_b200.roofline) on the CPU: the reference's
roofline functions keep their meaning (src/lws/domain/performance/
roofline.py:52-146), and the B200 calibration predicts the live per-GEMV
times measured on one B200 (bench.py's per_gemv, Gemma-2-2B decode-step
classes, batch 1) within max(15 %, 1.5 us) each."""

from __future__ import annotations

import pytest

from se12_b200 import roofline as rf

# (class, rows, cols, SE12 bytes, measured us per GEMV inside a stack of 26
# (1 for the LM head), 1 B200, 1965 MHz, one launch per GEMV)
MEASURED = [
    ("qkv_proj", 4096, 2304, 14.19e6, 7.83),
    ("o_proj", 2304, 2048, 7.10e6, 4.75),
    ("gate_up_proj", 18432, 2304, 63.87e6, 18.15),
    ("down_proj", 2304, 9216, 31.93e6, 12.66),
    ("lm_head", 256000, 2304, 887.06e6, 197.47),
]


def test_reference_functions_keep_their_meaning():
    w = 2304 * 9216
    mem = rf.memory_time(w, rf.bytes_per_weight(rf.WeightFormat.SE12), 6551.7)
    assert mem == pytest.approx(w * 12.03 / 8 / 6551.7e3)
    assert rf.memory_time(w, rf.bytes_per_weight(rf.WeightFormat.RAW_BF16), 1000.0) == pytest.approx(w * 2 / 1e6)
    # eta fitted from a latency is recovered by the prediction
    eta = rf.fit_overlap_efficiency(12.0, 10.0, 4.0)
    assert eta == pytest.approx(0.5)
    assert rf.predicted_latency(10.0, 4.0, eta) == pytest.approx(12.0)
    assert rf.fit_overlap_efficiency(5.0, 10.0, 4.0) == 1.0  # clamped
    assert rf.fit_overlap_efficiency(20.0, 10.0, 4.0) == 0.0
    # memory-bound with no compute: the ratio is the byte ratio
    assert rf.predict_shape_ratio(w, 6551.7, 0.0, 0.0, 1.0) == pytest.approx(12.03 / 16)


def test_fit_recovers_known_parameters():
    truth = rf.B200Calibration(hbm_gbs=6500.0, fixed_us=3.0, issue_us_per_tile=1.2e-3)
    samples = [(b, t, truth.gemv_us(b, t)) for b, t in ((7e6, 1152), (14e6, 2304), (64e6, 10368), (32e6, 5184),
                                                        (887e6, 144000))]
    fit = rf.fit_b200(samples, 6500.0)
    assert fit.fixed_us == pytest.approx(3.0, abs=0.05)
    assert fit.issue_us_per_tile == pytest.approx(1.2e-3, abs=2e-6)


@pytest.mark.parametrize("name,rows,cols,nbytes,us", MEASURED)
def test_b200_model_predicts_measured_gemv_times(name, rows, cols, nbytes, us):
    pred = rf.B200_DEFAULT.gemv_us(nbytes, rf.tiles_of(rows, cols))
    assert abs(pred - us) <= max(0.15 * us, 1.5), f"{name}: predicted {pred:.2f} us, measured {us:.2f} us"


def test_b200_default_is_the_fit_of_the_measurements():
    fit = rf.fit_b200([(b, rf.tiles_of(r, c), us) for _, r, c, b, us in MEASURED], rf.B200_DEFAULT.hbm_gbs)
    assert fit.fixed_us == pytest.approx(rf.B200_DEFAULT.fixed_us, abs=0.05)
    assert fit.issue_us_per_tile == pytest.approx(rf.B200_DEFAULT.issue_us_per_tile, rel=0.01)
