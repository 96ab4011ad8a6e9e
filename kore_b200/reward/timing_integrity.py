"""Timing-integrity taxonomy: the performance-hack classes a candidate can try
and the verifier defense that covers each (parity: kore/reward/timing_integrity.py)."""
from __future__ import annotations

from dataclasses import dataclass
from enum import Enum


class PerfHackClass(str, Enum):
    WARM_CACHE = "warm_cache"            # benefit from data left in L2 by the previous iteration
    DO_LESS_WORK = "do_less_work"        # skip work on timed iterations
    MODE_SNIFFING = "mode_sniffing"      # detect bench vs correctness mode
    ASYNC_ESCAPE = "async_escape"        # return before the GPU work finishes
    FORGED_TIMER = "forged_timer"        # print fake timing/verdict lines
    DELEGATION = "delegation"            # call cuBLAS / cuDNN / flashinfer / torch ops
    CACHED_OUTPUT = "cached_output"      # memoise results across calls
    NONDETERMINISM = "nondeterminism"    # random output that passes once by luck


@dataclass(frozen=True)
class Defense:
    name: str
    where: str


_COVERAGE = {
    PerfHackClass.WARM_CACHE: Defense("L2 flush (512 MiB write) before every timed iteration",
                                      "kore_b200.tasks.driver.l2_flush"),
    PerfHackClass.DO_LESS_WORK: Defense("post-timing re-verification of the output",
                                        "kore_b200.tasks.driver.run_bench"),
    PerfHackClass.MODE_SNIFFING: Defense("scanner bans argv/env/flag reads; randomised iteration counts",
                                         "kore_b200.reward.reward.scan_for_hacks"),
    PerfHackClass.ASYNC_ESCAPE: Defense("CUDA events on the launching stream + synchronize",
                                        "kore_b200.tasks.driver.time_events"),
    PerfHackClass.FORGED_TIMER: Defense("verdict parsed from the LAST matching line; scanner bans verdict prints",
                                        "kore_b200.env.kore_env"),
    PerfHackClass.DELEGATION: Defense("delegation regexes (vendor libs, torch ops, @)",
                                      "kore_b200.reward.reward.scan_for_hacks"),
    PerfHackClass.CACHED_OUTPUT: Defense("fresh random inputs per trial + output poisoning before calls",
                                         "kore_b200.tasks.driver.run_correctness"),
    PerfHackClass.NONDETERMINISM: Defense("determinism re-run with SNR tolerance",
                                          "kore_b200.env.kore_env.KoreEnv"),
}


def coverage():
    return dict(_COVERAGE)


def uncovered():
    return [c for c in PerfHackClass if c not in _COVERAGE]


def report() -> str:
    return "\n".join(f"{c.value:16s} -> {d.name} [{d.where}]" for c, d in _COVERAGE.items())
