"""Speed-of-light study runner with a fake driver (no GPU), replay mining,
the decision rule, and residual-model transfer across families."""
import json
import random

import pytest

from kore_b200.analysis import p0_runner as P
from kore_b200.analysis import residual_transfer as RT
from kore_b200.analysis.study import Record
from kore_b200.tasks.registry import get_task

PEAKS = {"hbm_bytes_per_s": 6.4e12, "bf16_flops_per_s": 1.6e15, "fp32_flops_per_s": 0.08e15,
         "fp16_flops_per_s": 1.6e15, "fp8_flops_per_s": 3.2e15}


def _fake_driver(cand_ms, ref_ms=1.0, snr=60.0):
    calls = []

    def run(cmd, cwd, timeout):
        calls.append(cmd)
        if "--bench-both" in cmd:
            return 0, f"CAND primary {cand_ms:.5f} 0.5\nREF primary {ref_ms:.5f} 0.4\nPOST_VERIFY_SNR primary 61\n"
        return 0, f"SNR: {snr:.2f} dB\nallclose: True\nmax_diff: 0.0001\n"
    return run, calls


def test_measure_kernel_with_fake_driver():
    t = get_task("gen_silu_bf16")
    sh = t.shape("primary") or t.shapes[0]
    run, calls = _fake_driver(0.5)
    m = P.measure_kernel(t, "seed", t.seed_src, sh, PEAKS, repeats=3, runner=run)
    assert m.correct and m.cand_ms == 0.5 and m.ref_ms == 1.0 and m.speedup == 2.0
    assert m.t_min_ms and 0 < m.eta < 10
    assert len(calls) == 4 and all("kore_b200.tasks.driver" in " ".join(c) for c in calls)
    bad, _ = _fake_driver(0.5, snr=5.0)
    assert not P.measure_kernel(t, "seed", t.seed_src, sh, PEAKS, runner=bad).correct


def test_trajectory_sources_are_distinct_and_start_with_the_seed():
    t = get_task("gen_silu_bf16")
    srcs = P.trajectory_sources(t, 4)
    assert srcs[0] == ("seed", t.seed_src)
    assert len({s for _, s in srcs}) == len(srcs)


def _records(seed=0):
    rng = random.Random(seed)
    rs = []
    for fam, scale in (("norm", 0.05), ("gemm", 1.0), ("attention", 0.5), ("reduce", 0.02)):
        for i in range(12):
            tmin = scale * (1 + rng.random())
            st, oc = tmin * rng.random(), tmin * rng.random() * 0.5
            t = tmin + 1.5 * st + 0.8 * oc + 0.01 * tmin * rng.random()
            rs.append(Record(f"{fam}_{i}", fam, tmin / t, 1.0 / t * tmin * 2, t, tmin, st, oc))
    return rs


def test_run_decide_and_render():
    ms = []
    for r in _records():
        ms.append(P.KernelMeasure(r.task_id, r.family, "k", "primary", True, 60.0, r.t_measured_ms,
                                  r.t_measured_ms * r.speedup, r.t_min_ms))
    rep = P.run(ms, iters=200)
    assert rep["n_records"] == len(ms) and rep["checks"]["a"]["verdict"] in ("PASS", "WEAK", "FAIL")
    assert rep["decision"].split(":")[0] in ("GO", "NO-GO", "CONDITIONAL")
    md = P.render(rep)
    assert "Spearman" in md and "| task |" in md
    assert P.run(ms[:2])["decision"].startswith("INSUFFICIENT")
    assert P.decide({k: {"verdict": "PASS"} for k in "abc"}).startswith("GO")
    assert P.decide({"a": {"verdict": "FAIL"}, "b": {"verdict": "PASS"}, "c": {"verdict": "PASS"}}).startswith("NO-GO")


def test_decompose_uses_counters():
    c = {"smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio": 3.0,
         "smsp__average_warps_issue_stalled_wait_per_issue_active.ratio": 1.0,
         "sm__warps_active.avg.pct_of_peak_sustained_active": 25.0}
    st, oc = P.decompose(c, 2.0, 1.0)
    assert st == pytest.approx(0.75) and oc == pytest.approx(0.75)


def test_replay_mining(tmp_path):
    from kore_b200.data.schemas import RankedGroupRecord
    rec = RankedGroupRecord("gen_silu_bf16", "p0", [{"source": "x", "correct": True, "wall_us": 50.0, "snr_db": 60},
                                                    {"source": "y", "correct": False}], [[0, 1]],
                            parent_wall_us=100.0)
    p = tmp_path / "g.jsonl"
    p.write_text(json.dumps(rec.to_dict()) + "\n")
    ms = P.mine_replay([str(p)], PEAKS)
    assert len(ms) == 2 and ms[0].speedup == 2.0 and not ms[1].correct


def test_residual_transfer():
    rs = _records()
    res = RT.run(rs)
    assert res["normalized"]["families"] == 4 and res["normalized"]["median_r2"] > 0.5
    assert res["verdict"].startswith("TRANSFERS")
    assert "held-out family" in RT.render(res)
    # families whose time depends on different residual terms do not transfer
    bad = []
    rng = random.Random(3)
    for fam, (a, b) in (("x", (3.0, 0.0)), ("y", (0.0, 3.0)), ("z", (-1.0, 0.0))):
        for i in range(10):
            st, oc = rng.random(), rng.random()
            bad.append(Record(f"{fam}{i}", fam, 0.5, 1.0, 1.0 + a * st + b * oc + 0.0, 1.0, st, oc))
    assert not RT.run(bad)["verdict"].startswith("TRANSFERS")
    dec = RT.family_decodability(rs)
    assert 0 <= dec["accuracy"] <= 1 and dec["chance"] == pytest.approx(0.25)


def test_study_figures_are_valid_svg(tmp_path):
    import xml.etree.ElementTree as ET

    from kore_b200.analysis import plots
    ms = []
    for r in _records():
        ms.append(P.KernelMeasure(r.task_id, r.family, "k", "primary", True, 60.0, r.t_measured_ms,
                                  r.t_measured_ms * r.speedup, r.t_min_ms))
    rep = json.loads(json.dumps(P.run(ms, iters=50), default=str))
    paths = plots.write_all(rep, str(tmp_path))
    assert len(paths) == 3
    for p in paths:
        root = ET.parse(p).getroot()
        assert root.tag.endswith("svg") and len(list(root.iter("{http://www.w3.org/2000/svg}circle"))) > 10
    empty = plots.scatter_svg({}, title="t", xlabel="x", ylabel="y")
    assert ET.fromstring(empty).tag.endswith("svg")


def test_study_cli_on_replayed_records(tmp_path):
    from kore_b200.data.schemas import RankedGroupRecord
    recs = []
    for i, tid in enumerate(["gen_silu_bf16", "gen_relu_bf16", "gen_add_bf16", "gen_mul_bf16", "gen_exp_bf16"]):
        recs.append(RankedGroupRecord(tid, "p", [{"source": "a", "correct": True, "wall_us": 40.0 + 5 * i},
                                                 {"source": "b", "correct": True, "wall_us": 80.0 + i}],
                                      [[0, 1]], parent_wall_us=100.0))
    p = tmp_path / "g.jsonl"
    p.write_text("\n".join(json.dumps(r.to_dict()) for r in recs) + "\n")
    out = tmp_path / "p0.json"
    assert P.main(["--replay", str(p), "--out", str(out), "--iters", "50"]) == 0
    rep = json.loads(out.read_text())
    assert rep["n_measured"] == 10 and rep["n_records"] == 10 and "checks" in rep
    assert (tmp_path / "p0.md").read_text().startswith("# Speed-of-light study")
    res = RT.run(RT.records_from_report(str(out)))
    assert "verdict" in res
