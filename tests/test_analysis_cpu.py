"""Speed-of-light study statistics on synthetic records with known structure."""
import random

from kore_b200.analysis.study import (Record, bottleneck_from_counters, leave_one_family_out, monotone_fraction,
                                      p0_checks, spearman)


def _records(n=120, seed=0):
    rng = random.Random(seed)
    out = []
    for i in range(n):
        fam = ["norm", "gemm", "attn"][i % 3]
        tmin = rng.uniform(0.01, 1.0)
        stall = rng.uniform(0, 0.5)
        occ = rng.uniform(0, 0.2)
        t = tmin + 0.8 * stall + 1.5 * occ + rng.gauss(0, 0.01)
        base = tmin * 2.0
        out.append(Record(f"t{i // 4}", fam, tmin / t, base / t, t, tmin, stall, occ))
    return out


def test_spearman_exact():
    assert spearman([1, 2, 3, 4], [10, 20, 30, 40]) == 1.0
    assert spearman([1, 2, 3, 4], [4, 3, 2, 1]) == -1.0


def test_p0_checks_pass_on_structured_data():
    rs = _records()
    r = p0_checks(rs, iters=200)
    assert r["a"]["spearman"] > 0.5 and r["a"]["verdict"] == "PASS"
    assert r["b"]["r2"] > 0.95 and r["b"]["verdict"] == "PASS"
    assert 0.0 <= monotone_fraction(rs) <= 1.0
    lofo = leave_one_family_out(rs)
    assert set(lofo) == {"norm", "gemm", "attn"} and min(lofo.values()) > 0.9


def test_bottleneck():
    assert bottleneck_from_counters({"sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active": 80,
                                     "gpu__time_duration.sum": 1e6}) == "tensor"
    assert bottleneck_from_counters({"gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed": 85,
                                     "gpu__time_duration.sum": 1e6}) == "dram"
    assert bottleneck_from_counters({"gpu__time_duration.sum": 2000}) == "launch"
