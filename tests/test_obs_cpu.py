"""Telemetry: events.jsonl schema, stage spans, per-thread stage stacks."""
import io
import json
import threading

import pytest

from kore_b200 import obs


def test_events_schema_and_spans(tmp_path):
    obs.configure(run_dir=tmp_path, level="DEBUG", color=False)
    buf = io.StringIO()
    old = obs.HUB.console.stream
    obs.HUB.console.stream = buf
    try:
        log = obs.get_logger("t")
        with log.stage("outer", n=1):
            log.info("hello", x=1.5)
            log.metric(loss=0.25)
        with pytest.raises(ValueError):
            with log.stage("bad"):
                raise ValueError("boom")
        seen = {}

        def worker():
            seen["stage"] = obs.get_logger("w").emit("INFO", "from thread")["stage"]

        with log.stage("main-only"):
            th = threading.Thread(target=worker)
            th.start()
            th.join()
    finally:
        obs.HUB.console.stream = old
    recs = [json.loads(l) for l in (tmp_path / "events.jsonl").read_text().splitlines()]
    for r in recs:
        assert {"ts", "elapsed_s", "level", "kind", "logger", "stage", "msg"} <= set(r)
    hello = next(r for r in recs if r["msg"] == "hello")
    assert hello["stage"] == "outer" and hello["fields"] == {"x": 1.5}
    assert any(r["kind"] == "stage" and r["level"] == "ERROR" and "boom" in r["fields"]["error"] for r in recs)
    assert seen["stage"] == "-"            # another thread is not inside the main thread's stage
    assert "hello" in buf.getvalue()


def test_phase_timer_cpu():
    pt = obs.PhaseTimer()
    with pt.phase("a"):
        pass
    with pt.phase("a"):
        pass
    out = pt.summary()
    assert set(out) == {"a"} and out["a"] >= 0.0
