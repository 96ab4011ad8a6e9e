"""Campaign orchestrator (manifest resume, stage skipping, failure record,
pause marker, retention hard stop), supervisor restart, LPT partition and
free-GPU picker against a fake NVML."""
import json
import sys
import types

import pytest


def _campaign(tmp_path, calls, fail=None):
    from kore_b200.campaign import orchestrator as o
    c = o.Campaign(tmp_path, "base-model", dry_run=True)

    def mk(st):
        def f(c, m):
            calls.append(st)
            if fail == st:
                raise RuntimeError("boom")
            return {"model": f"/m/{st}"} if st in o.TRAIN_STAGES else {}
        return f
    return o, c, {st: mk(st) for st in o.STAGES}


def test_manifest_resume_and_force(tmp_path, monkeypatch):
    calls = []
    o, c, fns = _campaign(tmp_path, calls)
    monkeypatch.setattr(o, "STAGE_FNS", fns)
    m = o.run(c)
    assert calls == [s for s in o.STAGES if s not in o.OPTIONAL_STAGES]
    assert all(v["status"] == "done" for v in m["stages"].values())
    calls.clear()
    o.run(c)
    assert calls == []                                   # everything resumed from the manifest
    o.run(c, force=["dpo"])
    assert calls == ["dpo"]                               # same outputs: downstream digests unchanged
    assert o._latest_model(c, json.loads(c.manifest_path.read_text())) == "/m/grpo"


def test_failure_recorded_then_resumes(tmp_path, monkeypatch):
    calls = []
    o, c, fns = _campaign(tmp_path, calls, fail="sft")
    monkeypatch.setattr(o, "STAGE_FNS", fns)
    with pytest.raises(RuntimeError):
        o.run(c)
    m = json.loads(c.manifest_path.read_text())
    assert m["stages"]["sft"]["status"] == "failed" and m["stages"]["midtrain"]["status"] == "done"
    calls.clear()
    o2, c2, fns2 = _campaign(tmp_path, calls)
    monkeypatch.setattr(o2, "STAGE_FNS", fns2)
    o2.run(c2)
    assert calls[0] == "sft"


def test_pause_marker(tmp_path, monkeypatch):
    from kore_b200.campaign.supervise import pause_after
    calls = []
    o, c, fns = _campaign(tmp_path, calls)
    monkeypatch.setattr(o, "STAGE_FNS", fns)
    pause_after(str(tmp_path), "datagen")
    m = o.run(c)
    assert calls == ["reverify", "datagen"] and m["paused_after"] == "datagen"


def test_retention_hard_stop(tmp_path, monkeypatch):
    calls = []
    o, c, fns = _campaign(tmp_path, calls)
    monkeypatch.setattr(o, "STAGE_FNS", fns)
    suite = tmp_path / "s.jsonl"
    suite.write_text(json.dumps({"prompt": "q", "answer": "yes"}) + "\n")
    c.retention_suites = {"toy": str(suite)}
    gen = lambda model: (lambda p: "yes" if model == "base-model" else "no")
    with pytest.raises(o.RetentionStop):
        o.run(c, generate_factory=gen)
    assert "eval" not in calls                           # stopped right after soup


def test_dry_run_launch_renders_config(tmp_path):
    from kore_b200.campaign import orchestrator as o
    c = o.Campaign(tmp_path, "base", gpus=2, dry_run=True)
    assert o.launch_stage(c, "sft", {"output_dir": "x"}) == 0
    assert json.loads((tmp_path / "sft" / "config.json").read_text())["output_dir"] == "x"


def test_supervisor_restarts(tmp_path):
    from kore_b200.campaign.supervise import supervise
    flag = tmp_path / "once"
    code = f"import os,sys\np={str(flag)!r}\nif not os.path.exists(p):\n    open(p,'w').close(); sys.exit(3)\n"
    import io
    out = io.StringIO()
    rc = supervise([sys.executable, "-c", code], max_restarts=2, heartbeat_s=5, backoff_s=0.01, out=out)
    assert rc == 0 and "ALERT exit=3" in out.getvalue()


def test_lpt_and_gpu_picker():
    from kore_b200.campaign.nodes import lpt_partition, pick_free_gpus
    parts = lpt_partition({"a": 7, "b": 5, "c": 4, "d": 3, "e": 3}, 2)
    loads = sorted(sum({"a": 7, "b": 5, "c": 4, "d": 3, "e": 3}[k] for k in p) for p in parts)
    assert loads == [10, 12]                             # LPT order; within 4/3 of the optimum 11

    class Mem:
        def __init__(self, u): self.used = u << 20
    usage = {0: (50000, 1), 1: (100, 0), 2: (10, 0), 3: (4096, 0)}
    fake = types.SimpleNamespace(
        nvmlInit=lambda: None, nvmlShutdown=lambda: None, nvmlDeviceGetCount=lambda: 4,
        nvmlDeviceGetHandleByIndex=lambda i: i, nvmlDeviceGetMemoryInfo=lambda h: Mem(usage[h][0]),
        nvmlDeviceGetComputeRunningProcesses=lambda h: [0] * usage[h][1])
    assert pick_free_gpus(2, nvml=fake) == [1, 2]
    with pytest.raises(RuntimeError):
        pick_free_gpus(3, nvml=fake, retries=2, sleep=lambda s: None)


def test_distill_sink_dedup(tmp_path):
    from kore_b200.policy.distill import DistillSink
    p = str(tmp_path / "wins.jsonl")
    s = DistillSink(p)
    assert s.add("t1", "src", 1.5, baseline_us=30.0)
    assert not s.add("t1", "src", 1.2)                  # worse duplicate dropped
    assert s.add("t1", "src", 2.0)
    assert not s.add("t2", "x", 0.9)                    # not a win
    assert s.flush() == 1
    s2 = DistillSink(p)
    assert len(s2.best) == 1 and list(s2.best.values())[0].speedup == 2.0


def test_iterative_dpo_stage_dry_run(tmp_path):
    from kore_b200.campaign.orchestrator import Campaign, run
    c = Campaign(out_dir=tmp_path, base_model="base", dry_run=True, configs={"dpo_iterative": {"rounds": 2}})
    m = run(c, stages=["dpo_iterative"])
    st = m["stages"]["dpo_iterative"]
    assert st["status"] == "done" and len(st["outputs"]["rounds"]) == 2
    assert st["outputs"]["model"].endswith("round1/model")
    cfg = (tmp_path / "dpo" / "config.json").read_text()
    assert "round0/model" in cfg and "ipo" in cfg          # round 2 trains from round 1's model
