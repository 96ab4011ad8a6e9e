"""Process supervisor and monitor for long campaigns.

``supervise(cmd)`` runs the campaign (or any stage command) in its own
process group, prints HEARTBEAT lines with elapsed time every
``heartbeat_s``, and on a non-zero exit relaunches it (the campaign resumes
from its manifest) up to ``max_restarts`` with backoff, printing ALERT lines.
It only ever signals the process group it started itself. ``monitor(dir)``
is read-only: it summarises the manifest and the tail of ``events.jsonl``.
``pause_after(stage)`` makes a campaign stop cleanly at a stage boundary.
Reference parity: scripts/kore_supervise.py:91-152, kore_monitor.py,
kore_pause_after_datagen.py, kore_resume_supervise.py.
"""
from __future__ import annotations

import argparse
import json
import os
import signal
import subprocess
import sys
import time
from pathlib import Path
from typing import List, Optional


def supervise(cmd: List[str], max_restarts: int = 5, heartbeat_s: float = 60.0, backoff_s: float = 10.0,
              out=sys.stdout) -> int:
    restarts = 0
    while True:
        t0 = time.time()
        p = subprocess.Popen(cmd, start_new_session=True)     # own process group, ours to signal
        try:
            while True:
                try:
                    rc = p.wait(timeout=heartbeat_s)
                    break
                except subprocess.TimeoutExpired:
                    print(f"HEARTBEAT pid={p.pid} elapsed_s={time.time() - t0:.0f}", file=out, flush=True)
        except KeyboardInterrupt:
            os.killpg(p.pid, signal.SIGTERM)
            p.wait()
            return 130
        if rc == 0:
            return 0
        restarts += 1
        print(f"ALERT exit={rc} restart={restarts}/{max_restarts}", file=out, flush=True)
        if restarts > max_restarts:
            return rc
        time.sleep(backoff_s * min(8, 2 ** (restarts - 1)))


def monitor(campaign_dir: str, tail: int = 10) -> dict:
    d = Path(campaign_dir)
    m = json.loads((d / "manifest.json").read_text()) if (d / "manifest.json").exists() else {"stages": {}}
    ev = []
    for p in (d / "events.jsonl", Path(os.environ.get("KORE_EVENTS", "")) if os.environ.get("KORE_EVENTS") else None):
        if p and p.exists():
            ev = [json.loads(l) for l in p.read_text().splitlines()[-tail:] if l.strip()]
            break
    return {"stages": {k: v.get("status") for k, v in m.get("stages", {}).items()}, "recent_events": ev}


def pause_after(campaign_dir: str, stage: str) -> None:
    """Marker read by the orchestrator between stages."""
    Path(campaign_dir, "PAUSE_AFTER").write_text(stage)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="kore supervise")
    ap.add_argument("--max-restarts", type=int, default=5)
    ap.add_argument("--heartbeat", type=float, default=60.0)
    ap.add_argument("--monitor", default="")
    ap.add_argument("cmd", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    if a.monitor:
        print(json.dumps(monitor(a.monitor), indent=2))
        return 0
    cmd = a.cmd[1:] if a.cmd and a.cmd[0] == "--" else a.cmd
    return supervise(cmd, a.max_restarts, a.heartbeat)


if __name__ == "__main__":
    raise SystemExit(main())
