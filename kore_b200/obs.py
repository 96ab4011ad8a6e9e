"""Structured logging for every stage: console lines + append-only JSONL.

Each record is ``{ts, elapsed_s, level, kind, logger, stage, msg, fields}``
(the reference's events.jsonl schema, kore/obs.py:110-113), written to
``<run_dir>/events.jsonl`` when a run directory is configured (``configure``
or ``KORE_RUN_DIR``). Helpers: log levels, ``event``, ``metric``, timed
``stage`` and ``timer`` contexts, ``progress`` with rate/ETA, ``heartbeat``
(adds GPU memory), and ``throughput`` (tokens/s with the max over ranks).
Stdlib only.
"""
from __future__ import annotations

import json
import os
import sys
import threading
import time
from contextlib import contextmanager
from pathlib import Path
from typing import Optional

LEVELS = {"DEBUG": 10, "INFO": 20, "WARN": 30, "WARNING": 30, "ERROR": 40}
_COLOR = {"DEBUG": "\033[2;37m", "INFO": "\033[0;36m", "WARN": "\033[0;33m", "ERROR": "\033[0;31m",
          "STAGE": "\033[1;35m", "METRIC": "\033[0;32m"}


class _RunState:
    def __init__(self):
        self.t0 = time.time()
        self.level = LEVELS.get(os.environ.get("KORE_LOG_LEVEL", "INFO").upper(), 20)
        self.stages: list = []
        self.lock = threading.RLock()
        self.path: Optional[Path] = None
        self.fh = None
        self.color = sys.stderr.isatty() and os.environ.get("KORE_LOG_COLOR", "1") != "0"
        if os.environ.get("KORE_RUN_DIR"):
            self.set_dir(os.environ["KORE_RUN_DIR"])

    def set_dir(self, d):
        with self.lock:
            p = Path(d)
            p.mkdir(parents=True, exist_ok=True)
            if self.fh:
                try:
                    self.fh.close()
                except OSError:
                    pass
            self.path = p / "events.jsonl"
            self.fh = self.path.open("a", encoding="utf-8")

    def write(self, rec: dict):
        with self.lock:
            if self.fh is not None:
                self.fh.write(json.dumps(rec, default=str) + "\n")
                self.fh.flush()


RUN = _RunState()


def configure(run_dir=None, level: Optional[str] = None, color: Optional[bool] = None) -> None:
    if run_dir is not None:
        RUN.set_dir(run_dir)
    if level is not None:
        RUN.level = LEVELS.get(level.upper(), RUN.level)
    if color is not None:
        RUN.color = bool(color)


def _hms(sec: float) -> str:
    sec = int(max(0, sec))
    h, r = divmod(sec, 3600)
    m, s = divmod(r, 60)
    return f"{h:d}:{m:02d}:{s:02d}" if h else f"{m:02d}:{s:02d}"


class KoreLogger:
    def __init__(self, name: str):
        self.name = name

    def _emit(self, level: str, msg: str, fields: dict, kind: str = "log") -> None:
        now = time.time()
        stage = RUN.stages[-1][0] if RUN.stages else "-"
        rec = {"ts": now, "elapsed_s": round(now - RUN.t0, 3), "level": level, "kind": kind,
               "logger": self.name, "stage": stage, "msg": msg}
        if fields:
            rec["fields"] = fields
        RUN.write(rec)
        if LEVELS.get(level, 20) < RUN.level:
            return
        tag = level if kind == "log" else kind.upper()
        line = f"[{_hms(now - RUN.t0)}] {tag:<6} {self.name}" + (f" ({stage})" if stage != "-" else "")
        line += f": {msg}"
        if fields:
            line += "  " + " ".join(f"{k}={v:.4g}" if isinstance(v, float) else f"{k}={v}"
                                    for k, v in fields.items())
        if RUN.color and tag in _COLOR:
            line = f"{_COLOR[tag]}{line}\033[0m"
        print(line, file=sys.stderr, flush=True)

    def debug(self, msg, **f): self._emit("DEBUG", msg, f)
    def info(self, msg, **f): self._emit("INFO", msg, f)
    def warn(self, msg, **f): self._emit("WARN", msg, f)
    warning = warn
    def error(self, msg, **f): self._emit("ERROR", msg, f)

    def event(self, name: str, **fields) -> None:
        self._emit("INFO", name, fields, kind="event")

    def metric(self, msg: str = "metrics", **kv) -> None:
        self._emit("INFO", msg, kv, kind="metric")

    @contextmanager
    def stage(self, name: str, **fields):
        RUN.stages.append((name, time.time()))
        self._emit("INFO", f"stage start: {name}", fields, kind="stage")
        t0 = time.time()
        try:
            yield self
        except Exception as e:
            self._emit("ERROR", f"stage FAILED: {name} ({type(e).__name__}: {e})",
                       {"elapsed_s": round(time.time() - t0, 2)}, kind="stage")
            raise
        else:
            self._emit("INFO", f"stage done: {name}", {"elapsed_s": round(time.time() - t0, 2), **fields},
                       kind="stage")
        finally:
            if RUN.stages:
                RUN.stages.pop()

    @contextmanager
    def timer(self, label: str, **fields):
        t0 = time.time()
        try:
            yield
        finally:
            self._emit("DEBUG", label, {"took_s": round(time.time() - t0, 3), **fields}, kind="timer")

    def progress(self, i: int, n: int, label: str = "", *, t_start: Optional[float] = None, **fields):
        extra = {}
        if t_start is not None and i > 0:
            rate = i / max(time.time() - t_start, 1e-9)
            extra = {"rate_per_s": round(rate, 3), "eta": _hms((n - i) / rate) if rate > 0 else "inf"}
        pct = 100.0 * i / n if n else 0.0
        self._emit("INFO", f"{label} {i}/{n} ({pct:.0f}%)", {**extra, **fields}, kind="progress")

    def heartbeat(self, label: str = "alive", **fields) -> None:
        fields.update(gpu_mem_snapshot())
        self._emit("DEBUG", label, fields, kind="heartbeat")

    def throughput(self, label: str, tokens: int, seconds_max_over_ranks: float, **fields):
        tps = tokens / max(seconds_max_over_ranks, 1e-12)
        self._emit("INFO", label, {"tokens": tokens, "seconds": seconds_max_over_ranks,
                                   "tokens_per_s": tps, **fields}, kind="metric")
        return tps


def get_logger(name: str) -> KoreLogger:
    return KoreLogger(name)


def gpu_mem_snapshot() -> dict:
    try:
        import torch
        if not torch.cuda.is_available():
            return {}
        return {f"gpu{i}_gb": round(torch.cuda.max_memory_allocated(i) / 1e9, 2)
                for i in range(torch.cuda.device_count())}
    except Exception:  # noqa: BLE001 - best effort only
        return {}


class PhaseTimer:
    """Per-phase device time of a training step (rollout / logp / fwd-bwd /
    optimizer / sync): each phase is an NVTX range (visible in any CUDA
    profiler timeline) bracketed by CUDA events on the current stream.
    ``summary(ctx)`` synchronises once and returns milliseconds per phase,
    max over ranks. On CPU it falls back to wall time."""

    def __init__(self, enabled: bool = True):
        import torch
        self.cuda = enabled and torch.cuda.is_available()
        self.spans = []

    @contextmanager
    def phase(self, name: str):
        import torch
        if self.cuda:
            torch.cuda.nvtx.range_push(name)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            try:
                yield
            finally:
                e.record()
                torch.cuda.nvtx.range_pop()
                self.spans.append((name, s, e))
        else:
            t0 = time.time()
            try:
                yield
            finally:
                self.spans.append((name, t0, time.time()))

    def summary(self, ctx=None) -> dict:
        import torch
        out: dict = {}
        if self.cuda:
            torch.cuda.synchronize()
        for name, s, e in self.spans:
            ms = s.elapsed_time(e) if self.cuda else (e - s) * 1e3
            out[name] = out.get(name, 0.0) + ms
        if ctx is not None and getattr(ctx, "enabled", False):
            out = {k: ctx.max_over_ranks(v) for k, v in sorted(out.items())}
        self.spans = []
        return out
