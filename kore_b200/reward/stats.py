"""Timing statistics (median / mean / population std / coefficient of variation)."""
from __future__ import annotations

import math


def median(xs):
    s = sorted(xs)
    n = len(s)
    if n == 0:
        return float("nan")
    return s[n // 2] if n % 2 else 0.5 * (s[n // 2 - 1] + s[n // 2])


def mean(xs):
    return sum(xs) / len(xs) if xs else float("nan")


def std(xs):
    if len(xs) < 2:
        return 0.0
    m = mean(xs)
    return math.sqrt(sum((x - m) ** 2 for x in xs) / len(xs))


def cv_pct(xs):
    m = mean(xs)
    return 100.0 * std(xs) / m if xs and m else float("nan")
