"""Failure detection between steps: heartbeats in the rendezvous store.

Every rank publishes ``hb/<rank> = (step, wall time)`` into a key-value
store (the torch.distributed TCPStore of the job, or any ``Store``) after
each step, and, before launching its next step's kernels and collectives,
checks that every peer reached the previous step within ``timeout_s``.
A rank that died, exited or never joined is reported as a
:class:`PeerFailure` on the host, so survivors stop between steps instead of
entering a collective that would hang; the supervisor then relaunches the
job from its last checkpoint. A rank leaving cleanly marks itself ``left``.

``classify_exception`` maps failures to the reward / retry taxonomy: infra
(timeouts, OOM, lost peers, NCCL errors; retried, never trained on) versus
program errors. Reference parity: kore/env/kore_env.py:80-86 and :276-288
(infra classification), scripts/kore_supervise.py:133-152 (relaunch); the
reference has no heartbeat, this is the B200 plan's host-side detection.
"""
from __future__ import annotations

import json
import time
from typing import Callable, List, Optional


class PeerFailure(RuntimeError):
    def __init__(self, ranks: List[int], detail: str):
        super().__init__(f"peer ranks {ranks} failed: {detail}")
        self.ranks = ranks


class Heartbeat:
    def __init__(self, store, rank: int, world: int, timeout_s: float = 60.0,
                 clock: Callable[[], float] = time.time, poll_s: float = 0.05):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.clock, self.poll_s = timeout_s, clock, poll_s
        self.step = -1

    def _key(self, r: int) -> str:
        return f"kore/hb/{r}"

    def beat(self, step: int) -> None:
        self.step = step
        self.store.set(self._key(self.rank), json.dumps({"step": step, "t": self.clock()}))

    def leave(self) -> None:
        self.store.set(self._key(self.rank), json.dumps({"step": self.step, "t": self.clock(), "left": True}))

    def _read(self, r: int) -> Optional[dict]:
        try:
            if hasattr(self.store, "check") and not self.store.check([self._key(r)]):
                return None
            return json.loads(self.store.get(self._key(r)))
        except Exception:  # noqa: BLE001 - missing key / store gone counts as no heartbeat
            return None

    def wait_peers(self, step: int) -> None:
        """Block until every peer has published ``step`` (or later); raise
        PeerFailure for peers that left or stayed silent for timeout_s."""
        t0 = self.clock()
        while True:
            missing, left = [], []
            for r in range(self.world):
                if r == self.rank:
                    continue
                d = self._read(r)
                if d is not None and d.get("left"):
                    left.append(r)
                elif d is None or d["step"] < step:
                    missing.append(r)
            if left:
                raise PeerFailure(left, "left the job")
            if not missing:
                return
            if self.clock() - t0 > self.timeout_s:
                raise PeerFailure(missing, f"no heartbeat for step {step} within {self.timeout_s}s")
            time.sleep(self.poll_s)


def classify_exception(e: BaseException) -> str:
    """'infra' (retry, never train on) or 'program'."""
    if isinstance(e, (PeerFailure, TimeoutError, MemoryError)):
        return "infra"
    s = f"{type(e).__name__}: {e}".lower()
    for pat in ("out of memory", "nccl", "timed out", "timeout", "connection reset", "broken pipe",
                "device-side", "cuda error", "peer", "socket"):
        if pat in s:
            return "infra"
    return "program"


def guarded_steps(step_fn: Callable[[int], object], hb: Heartbeat, steps: int, start: int = 0):
    """Run ``step_fn(i)`` for i in [start, steps) with a heartbeat before and
    after each step; returns the list of results. Raises PeerFailure between
    steps when a peer is gone."""
    out = []
    for i in range(start, steps):
        hb.wait_peers(i - 1) if i > start else None
        out.append(step_fn(i))
        hb.beat(i)
    return out
