"""Performance model of the fused SE12 GEMV, recalibrated to B200.

The reference's roofline (src/lws/domain/performance/roofline.py:52-146)
predicts a GEMV's latency from its weight count alone:

    t_mem     = bytes_per_weight . W / BW
    t_compute = W . c(format)
    t         = max(t_mem, t_compute) + (1 - eta) . min(t_mem, t_compute)

with eta fitted once per GPU from a measured raw-kernel latency. The same
functions are kept here (same names, arguments and meaning) so callers of
the reference's model find them.

On B200 that model misses the term that decides the small projections of a
decode step: every dependent GEMV pays a fixed cost (its grid filling,
draining and handing over to the next kernel), about as long as the data
time of a 2304 x 2048 projection. ``B200Calibration`` therefore models one
GEMV of this package's kernel as

    t = t_fixed + max(t_mem, t_issue) + (1 - eta) . min(t_mem, t_issue)

where t_mem = SE12 bytes / measured HBM bandwidth (MEASURED_PEAKS.json's
copy rate) and t_issue = tiles . issue cost per tile (the kernel is bound
by its integer pipe on large matrices: a 16 x 256 tile costs a fixed
number of warp instructions to decode and multiply). ``fit_b200`` fits
t_fixed and the per-tile cost by least squares on measured live times
(``bench.py`` reports them per GEMV class as ``per_gemv``), with eta = 1:
on B200 the weight stream and the decode overlap fully (the pipeline keeps
several stages of copies in flight while the consumer warps decode).
"""

from __future__ import annotations

import dataclasses
import enum
import math

SE12_BYTES_PER_WEIGHT = 12.03 / 8  # the reference's design figure (roofline.py:23)
RAW_BYTES_PER_WEIGHT = 2.0
BYTES_PER_US_PER_GBS = 1000.0  # 1 GB/s = 1e9 B/s = 1e3 B/us
TILE_WEIGHTS = 16 * 256


class WeightFormat(enum.Enum):
    RAW_BF16 = "raw_bf16"
    SE12 = "se12"


def bytes_per_weight(weight_format: WeightFormat) -> float:
    """roofline.py:40-43."""
    return SE12_BYTES_PER_WEIGHT if weight_format is WeightFormat.SE12 else RAW_BYTES_PER_WEIGHT


def memory_time(weight_count: int, format_bytes: float, bandwidth_gbs: float) -> float:
    """Microseconds to stream ``weight_count`` weights at ``format_bytes``
    each over ``bandwidth_gbs`` (roofline.py:52-60)."""
    return weight_count * format_bytes / (bandwidth_gbs * BYTES_PER_US_PER_GBS)


def compute_time(weight_count: int, cost_us_per_weight: float) -> float:
    """roofline.py:63-67."""
    return weight_count * cost_us_per_weight


def fit_overlap_efficiency(measured_us: float, mem_us: float, compute_us: float) -> float:
    """eta in [0, 1] solving measured = max + (1 - eta) . min
    (roofline.py:77-91)."""
    larger, smaller = max(mem_us, compute_us), min(mem_us, compute_us)
    if smaller <= 0:
        return 1.0
    eta = 1.0 - (measured_us - larger) / smaller
    return min(max(eta, 0.0), 1.0)


def predicted_latency(mem_us: float, compute_us: float, overlap: float) -> float:
    """roofline.py:94-102."""
    return max(mem_us, compute_us) + (1.0 - overlap) * min(mem_us, compute_us)


def predict_ratio(fused_us: float, baseline_us: float) -> float:
    """roofline.py:110-114."""
    return fused_us / baseline_us


def predict_shape_ratio(weight_count: int, bandwidth_gbs: float, raw_cost: float, se12_cost: float,
                        overlap: float) -> float:
    """Fused / raw latency ratio from a shape and one GPU's calibration
    (roofline.py:132-146)."""
    raw = predicted_latency(memory_time(weight_count, RAW_BYTES_PER_WEIGHT, bandwidth_gbs),
                            compute_time(weight_count, raw_cost), overlap)
    se12 = predicted_latency(memory_time(weight_count, SE12_BYTES_PER_WEIGHT, bandwidth_gbs),
                             compute_time(weight_count, se12_cost), overlap)
    return predict_ratio(se12, raw)


# ------------------------------------------------------------------ B200


@dataclasses.dataclass(frozen=True)
class B200Calibration:
    """One GPU's calibration of this package's fused GEMV."""

    hbm_gbs: float            # measured copy bandwidth (MEASURED_PEAKS.json hbm_gbs)
    fixed_us: float           # per dependent launch: fill, drain, hand-over
    issue_us_per_tile: float  # integer-pipe cost of one 16 x 256 tile, over the whole GPU
    overlap: float = 1.0

    def gemv_us(self, se12_bytes: float, tiles: int) -> float:
        """Predicted live time of one GEMV (batch 1) inside a stack of GEMVs."""
        mem = se12_bytes / (self.hbm_gbs * BYTES_PER_US_PER_GBS)
        issue = tiles * self.issue_us_per_tile
        return self.fixed_us + predicted_latency(mem, issue, self.overlap)

    def roofline_fraction(self, se12_bytes: float, tiles: int) -> float:
        """Predicted fraction of the copy roofline one GEMV reaches."""
        return se12_bytes / (self.hbm_gbs * BYTES_PER_US_PER_GBS) / self.gemv_us(se12_bytes, tiles)


# Fitted (fit_b200) on live per-GEMV times of the Gemma-2-2B decode step's
# classes at batch 1 on one B200 (bench.py's per_gemv: q/k/v grouped, o,
# gate/up grouped, down, lm_head; 1965 MHz) against the measured copy rate.
B200_DEFAULT = B200Calibration(hbm_gbs=6551.7, fixed_us=4.49, issue_us_per_tile=1.34e-3)


def tiles_of(rows: int, cols: int) -> int:
    return math.ceil(rows / 16) * math.ceil(cols / 256)


def fit_b200(samples, hbm_gbs: float) -> B200Calibration:
    """Least-squares fit of the fixed cost and the per-tile issue cost from
    measured live times. ``samples``: (se12_bytes, tiles, measured_us) per
    GEMV class. With eta = 1 the model is t = f + max(m, c . tiles): for a
    given c the best f is the mean residual, so the fit scans c (1 ns to
    4 us per tile, 1 ns steps) and keeps the pair with the least squared
    error."""
    samples = [(float(b), int(t), float(us)) for b, t, us in samples]
    if len(samples) < 2:
        raise ValueError("need at least two GEMV classes to fit")
    bw = hbm_gbs * BYTES_PER_US_PER_GBS
    best = None
    for k in range(1, 4001):
        c = k * 1e-6  # us per tile, 1e-6 .. 4e-3
        # f minimises sum (us - f - max(m, c t))^2 for this c
        resid = [us - max(b / bw, c * t) for b, t, us in samples]
        f = sum(resid) / len(resid)
        err = sum((r - f) ** 2 for r in resid)
        if best is None or err < best[0]:
            best = (err, f, c)
    _, f, c = best
    return B200Calibration(hbm_gbs=hbm_gbs, fixed_us=max(f, 0.0), issue_us_per_tile=c)


__all__ = [
    "B200Calibration", "B200_DEFAULT", "RAW_BYTES_PER_WEIGHT", "SE12_BYTES_PER_WEIGHT", "WeightFormat", "bytes_per_weight",
    "compute_time", "fit_b200", "fit_overlap_efficiency", "memory_time", "predict_ratio", "predict_shape_ratio",
    "predicted_latency", "tiles_of",
]
