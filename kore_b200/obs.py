"""Run telemetry: a fan-out of structured records to pluggable sinks.

Design. Every log call builds one record and hands it to each registered
sink. Two sinks ship: ``JsonlSink`` (append-only ``events.jsonl``, one JSON
object per line) and ``ConsoleSink`` (a compact human line on stderr). A
sink decides on its own whether a record passes its level; the JSONL sink
keeps everything, so a post-mortem sees DEBUG records that the console hid.

Record schema (an interface: dashboards and monitors written against the
reference read the same file, kore/obs.py:110-113)::

    {"ts", "elapsed_s", "level", "kind", "logger", "stage", "msg", "fields"?}

Stages are spans kept on a per-thread stack, so a data-loader thread that
logs does not appear inside the trainer's stage. ``PhaseTimer`` is the
device-side counterpart: NVTX ranges plus CUDA events per training phase,
reduced as the max over ranks.

Environment: ``KORE_RUN_DIR`` (attach a JSONL sink there at import),
``KORE_LOG_LEVEL`` (console threshold), ``KORE_LOG_COLOR=0`` (plain console).
Stdlib only at import time.
"""
from __future__ import annotations

import json
import os
import sys
import threading
import time
from contextlib import contextmanager
from pathlib import Path
from typing import Callable, Dict, List, Optional

_RANK = {"DEBUG": 10, "INFO": 20, "WARN": 30, "WARNING": 30, "ERROR": 40}


def _level_no(name: Optional[str], default: int = 20) -> int:
    return _RANK.get((name or "").upper(), default)


# ----------------------------------------------------------------------------- sinks

class JsonlSink:
    """Appends every record to ``<dir>/events.jsonl`` (line-buffered)."""

    def __init__(self, run_dir):
        self.dir = Path(run_dir)
        self.dir.mkdir(parents=True, exist_ok=True)
        self.path = self.dir / "events.jsonl"
        self._fh = open(self.path, "a", encoding="utf-8", buffering=1)

    def __call__(self, rec: dict) -> None:
        self._fh.write(json.dumps(rec, default=str, separators=(",", ":")) + "\n")

    def close(self) -> None:
        try:
            self._fh.close()
        except OSError:
            pass


class ConsoleSink:
    """``+<seconds>s L logger[stage] msg | k=v ...`` on a text stream."""

    _TINT = {10: "2", 20: "0", 30: "33", 40: "1;31"}

    def __init__(self, stream=None, level: int = 20, color: Optional[bool] = None):
        self.stream = stream or sys.stderr
        self.level = level
        if color is None:
            color = getattr(self.stream, "isatty", lambda: False)() and os.environ.get("KORE_LOG_COLOR", "1") != "0"
        self.color = color

    @staticmethod
    def _fmt(v) -> str:
        if isinstance(v, float):
            return f"{v:.4g}"
        return str(v)

    def __call__(self, rec: dict) -> None:
        lv = _level_no(rec["level"])
        if lv < self.level:
            return
        where = rec["logger"] if rec["stage"] == "-" else f"{rec['logger']}[{rec['stage']}]"
        kind = "" if rec["kind"] == "log" else f"<{rec['kind']}> "
        text = f"+{rec['elapsed_s']:.1f}s {rec['level'][0]} {where} {kind}{rec['msg']}"
        if rec.get("fields"):
            text += " | " + " ".join(f"{k}={self._fmt(v)}" for k, v in rec["fields"].items())
        if self.color:
            text = f"\033[{self._TINT.get(lv, '0')}m{text}\033[0m"
        print(text, file=self.stream, flush=True)


# ----------------------------------------------------------------------------- hub

class Telemetry:
    """Holds the run clock, the sinks and the per-thread stage stacks."""

    def __init__(self):
        self.t0 = time.time()
        self.console = ConsoleSink(level=_level_no(os.environ.get("KORE_LOG_LEVEL"), 20))
        self.jsonl: Optional[JsonlSink] = None
        self.extra: List[Callable[[dict], None]] = []
        self._lock = threading.Lock()
        self._tls = threading.local()
        if os.environ.get("KORE_RUN_DIR"):
            self.attach_dir(os.environ["KORE_RUN_DIR"])

    # per-thread stage stack
    def stack(self) -> list:
        s = getattr(self._tls, "stack", None)
        if s is None:
            s = self._tls.stack = []
        return s

    def attach_dir(self, run_dir) -> Path:
        with self._lock:
            if self.jsonl is not None:
                self.jsonl.close()
            self.jsonl = JsonlSink(run_dir)
            return self.jsonl.path

    def publish(self, rec: dict) -> None:
        with self._lock:
            sinks = [s for s in (self.jsonl, self.console) if s is not None] + list(self.extra)
            for s in sinks:
                try:
                    s(rec)
                except Exception:  # noqa: BLE001 - a broken sink never stops training
                    pass


HUB = Telemetry()


def configure(run_dir=None, level: Optional[str] = None, color: Optional[bool] = None) -> None:
    """Attach a JSONL sink under ``run_dir`` and/or change the console level/colour."""
    if run_dir is not None:
        HUB.attach_dir(run_dir)
    if level is not None:
        HUB.console.level = _level_no(level, HUB.console.level)
    if color is not None:
        HUB.console.color = bool(color)


def add_sink(fn: Callable[[dict], None]) -> Callable[[], None]:
    """Register an extra sink (e.g. a metrics exporter); returns its remover."""
    HUB.extra.append(fn)
    return lambda: HUB.extra.remove(fn) if fn in HUB.extra else None


def events_path() -> Optional[Path]:
    return HUB.jsonl.path if HUB.jsonl is not None else None


def _clock(sec: float) -> str:
    sec = max(0, int(sec))
    return "%d:%02d:%02d" % (sec // 3600, sec % 3600 // 60, sec % 60)


# ----------------------------------------------------------------------------- logger

class KoreLogger:
    """A named emitter. ``kind`` tags the record: log, event, metric, stage,
    timer, progress or heartbeat."""

    def __init__(self, name: str):
        self.name = name

    def emit(self, level: str, msg: str, fields: Optional[Dict] = None, kind: str = "log") -> dict:
        now = time.time()
        st = HUB.stack()
        rec = {"ts": now, "elapsed_s": round(now - HUB.t0, 3), "level": level.upper(), "kind": kind,
               "logger": self.name, "stage": st[-1] if st else "-", "msg": msg}
        if fields:
            rec["fields"] = dict(fields)
        HUB.publish(rec)
        return rec

    def debug(self, msg, **f):
        self.emit("DEBUG", msg, f)

    def info(self, msg, **f):
        self.emit("INFO", msg, f)

    def warn(self, msg, **f):
        self.emit("WARN", msg, f)

    warning = warn

    def error(self, msg, **f):
        self.emit("ERROR", msg, f)

    def event(self, name: str, **fields) -> None:
        self.emit("INFO", name, fields, kind="event")

    def metric(self, msg: str = "metrics", **kv) -> None:
        self.emit("INFO", msg, kv, kind="metric")

    @contextmanager
    def stage(self, name: str, **fields):
        """A span: one record on entry, one on exit (``ok`` or ``error``), with
        its duration; nested spans show the innermost name in ``stage``."""
        st = HUB.stack()
        st.append(name)
        begin = time.time()
        self.emit("INFO", f"{name}: begin", fields, kind="stage")
        try:
            yield self
        except BaseException as exc:
            self.emit("ERROR", f"{name}: error", {"error": f"{type(exc).__name__}: {exc}",
                                                   "elapsed_s": round(time.time() - begin, 3)}, kind="stage")
            raise
        else:
            self.emit("INFO", f"{name}: ok", {**fields, "elapsed_s": round(time.time() - begin, 3)},
                      kind="stage")
        finally:
            if st and st[-1] == name:
                st.pop()

    span = stage

    @contextmanager
    def timer(self, label: str, **fields):
        begin = time.perf_counter()
        try:
            yield
        finally:
            self.emit("DEBUG", label, {**fields, "took_s": round(time.perf_counter() - begin, 4)}, kind="timer")

    def progress(self, i: int, n: int, label: str = "", *, t_start: Optional[float] = None, **fields):
        f = dict(fields)
        f["done"], f["total"] = i, n
        if t_start is not None and i > 0:
            dt = max(time.time() - t_start, 1e-9)
            rate = i / dt
            f["rate_per_s"] = round(rate, 3)
            f["eta"] = _clock((n - i) / rate) if rate > 0 else "inf"
        self.emit("INFO", f"{label} {100.0 * i / n if n else 0.0:.0f}%".strip(), f, kind="progress")

    def heartbeat(self, label: str = "alive", **fields) -> None:
        self.emit("DEBUG", label, {**fields, **gpu_mem_snapshot()}, kind="heartbeat")

    def throughput(self, label: str, tokens: int, seconds_max_over_ranks: float, **fields) -> float:
        tps = tokens / max(seconds_max_over_ranks, 1e-12)
        self.emit("INFO", label, {"tokens": tokens, "seconds": seconds_max_over_ranks,
                                  "tokens_per_s": tps, **fields}, kind="metric")
        return tps


_LOGGERS: Dict[str, KoreLogger] = {}


def get_logger(name: str) -> KoreLogger:
    lg = _LOGGERS.get(name)
    if lg is None:
        lg = _LOGGERS[name] = KoreLogger(name)
    return lg


def gpu_mem_snapshot() -> dict:
    """Peak allocated GB per visible GPU (empty without CUDA)."""
    torch = sys.modules.get("torch")
    try:
        if torch is None or not torch.cuda.is_available():
            return {}
        return {f"gpu{i}_gb": round(torch.cuda.max_memory_allocated(i) / 1e9, 2)
                for i in range(torch.cuda.device_count())}
    except Exception:  # noqa: BLE001
        return {}


# ----------------------------------------------------------------------------- device phases

class PhaseTimer:
    """Device time per phase of a training step.

    Each ``phase(name)`` is an NVTX range bracketed by two CUDA events on the
    current stream; nothing synchronises until ``summary``, which sums the
    phases by name and, given a distributed context, reduces each to its max
    over ranks. Without CUDA the phases are wall-clock."""

    def __init__(self, enabled: bool = True):
        import torch
        self._torch = torch
        self.cuda = bool(enabled) and torch.cuda.is_available()
        self.spans: list = []

    @contextmanager
    def phase(self, name: str):
        torch = self._torch
        if not self.cuda:
            begin = time.perf_counter()
            try:
                yield
            finally:
                self.spans.append((name, (time.perf_counter() - begin) * 1e3))
            return
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push(name)
        a.record()
        try:
            yield
        finally:
            b.record()
            torch.cuda.nvtx.range_pop()
            self.spans.append((name, (a, b)))

    def summary(self, ctx=None) -> dict:
        if self.cuda:
            self._torch.cuda.synchronize()
        out: dict = {}
        for name, v in self.spans:
            ms = v[0].elapsed_time(v[1]) if isinstance(v, tuple) else v
            out[name] = out.get(name, 0.0) + ms
        self.spans = []
        if ctx is not None and getattr(ctx, "enabled", False):
            out = {k: ctx.max_over_ranks(out[k]) for k in sorted(out)}
        return out
