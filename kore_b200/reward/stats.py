"""Timing statistics for the bench loop: median, mean, sample standard
deviation and coefficient of variation.

The CV gates the fast_p bonus (CV <= 3 %), so its estimator matters on the
3-5 run timings the environment takes: the spread is the unbiased sample
variance (divide by n - 1), as in kore/reward/stats.py:23-28, and an empty or
zero-mean series has an infinite CV (never trusted)."""
from __future__ import annotations

import math
import statistics


def median(xs):
    if not xs:
        return float("nan")
    return float(statistics.median(xs))


def mean(xs):
    return math.fsum(xs) / len(xs) if xs else float("nan")


def std(xs):
    """Sample standard deviation; 0 for fewer than two values."""
    return float(statistics.stdev(xs)) if len(xs) >= 2 else 0.0


def cv_pct(xs):
    m = mean(xs)
    if not xs or m == 0 or math.isnan(m):
        return float("inf")
    return 100.0 * std(xs) / abs(m)
