"""Re-verification of stored records with a fake environment: groups are
re-ranked, stale wins and repairs dropped, and a re-run resumes."""
from types import SimpleNamespace

from kore_b200.data import reverify as R
from kore_b200.data.schemas import RankedGroupRecord, RepairRecord, WinRecord, read_records, write_records

SEED = "def f(x):\n    return x\n"


class FakeEnv:
    """wall time (ms) by source; sources containing 'bad' fail correctness."""

    def __init__(self, walls):
        self.task = SimpleNamespace(seed_src=SEED, task_id="t")
        self.walls = walls
        self.calls = 0

    def step(self, src):
        self.calls += 1
        bad = "bad" in src
        return SimpleNamespace(compiled=True, validation_passed=not bad, wall_ms=None if bad else self.walls.get(src, 1.0),
                               snr_db=-5.0 if bad else 60.0)


def _kernel_msg(src):
    return {"role": "assistant", "content": "ANALYSIS: a\nPROPOSED_CHANGE: b\nFULL_KERNEL:\n```python\n" + src + "```\n"}


def test_group_is_reranked_and_prefs_rebuilt():
    env = FakeEnv({SEED: 1.0, "a": 0.5, "b": 0.8, "c": 0.81})
    rec = RankedGroupRecord("t", "p", [{"source": "b", "correct": True, "wall_us": 100},
                                       {"source": "a", "correct": True, "wall_us": 900},
                                       {"source": "bad", "correct": True, "wall_us": 10},
                                       {"source": "c", "correct": True, "wall_us": 5}], [[3, 2]])
    new = R.reverify_group(rec, env)
    assert [c["rank"] for c in new.candidates] == [1, 0, 3, 2]
    assert new.preferences == [[1, 0], [3, 2]]           # b vs c within the 2% margin: no pair
    assert new.candidates[2]["correct"] is False and new.parent_wall_us == 1000.0
    assert R.reverify_group(RankedGroupRecord("t", "p", [{"source": "bad"}], []), env) is None


def test_wins_and_repairs():
    env = FakeEnv({SEED: 1.0, "fast": 0.5, "slow": 1.2})
    w = WinRecord("t", [_kernel_msg("fast")], 10.0, 1.0, 10.0)
    nw = R.reverify_win(w, env)
    assert nw.speedup == 2.0 and nw.final_wall_us == 500.0 and nw.final_kernel.strip() == "fast"
    assert R.reverify_win(WinRecord("t", [], 1, 1, 1, final_kernel="slow"), env) is None
    assert R.reverify_win(WinRecord("t", [], 1, 1, 1, final_kernel="bad"), env) is None
    rp = RepairRecord("t", "snr_fail", "h", "e", [{"role": "user", "content": "fix"}, _kernel_msg("ok")])
    assert R.reverify_repair(rp, env).child_snr_db == 60.0
    rp2 = RepairRecord("t", "snr_fail", "h", "e", [_kernel_msg("bad")])
    assert R.reverify_repair(rp2, env) is None


def test_file_reverify_resumes(tmp_path):
    src = tmp_path / "in.jsonl"
    write_records(src, [WinRecord("t", [], 1, 1, 1, final_kernel="fast"),
                        WinRecord("t", [], 1, 1, 1, final_kernel="slow"),
                        RepairRecord("t", "c", "h", "e", [_kernel_msg("ok")]),
                        RankedGroupRecord("missing_task", "p", [{"source": "a"}], [])])
    env = FakeEnv({SEED: 1.0, "fast": 0.5, "slow": 2.0})

    def factory(tid):
        if tid != "t":
            raise KeyError(tid)
        return env
    out = str(tmp_path / "out.jsonl")
    st = R.reverify_file([str(src)], out, factory)
    assert st == {"seen": 4, "kept": 2, "dropped": 2, "skipped": 0}
    assert len(list(read_records(out))) == 2
    n = env.calls
    st2 = R.reverify_file([str(src)], out, factory)
    assert st2["skipped"] == 4 and env.calls == n and len(list(read_records(out))) == 2
    assert R.reverify_file([str(src)], str(tmp_path / "w.jsonl"), factory, kind="wins")["seen"] == 2


def test_rigorous_env_restores():
    import os
    before = os.environ.get("KORE_CORRECTNESS_TRIALS")
    with R.rigorous_env(17):
        assert os.environ["KORE_CORRECTNESS_TRIALS"] == "17"
    assert os.environ.get("KORE_CORRECTNESS_TRIALS") == before
