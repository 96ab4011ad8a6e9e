"""Agentic tool-use and kernel-QA data generators (reference parity:
kore/data/gen_agentic.py:81, gen_qa.py:212): the teacher drives the tool
harness (build/test/bench/pmc) on a task; trajectories that end with a
verified kernel are kept as chat rows; QA rows pair a kernel-engineering
question about a task with the teacher's answer."""
from __future__ import annotations

from typing import List

from .datasets import write_jsonl


def main(kind: str, tasks, teacher, env_factory, out: str) -> int:
    rows: List[dict] = []
    if kind == "agentic":
        from ..agent.harness import AgentHarness
        for t in tasks:
            h = AgentHarness(env_factory(t), t, max_turns=6)
            ep = h.run(teacher)
            if ep.best_correct:
                rows.append({"messages": ep.messages, "_source": "agentic", "task_id": t.task_id})
    else:
        for t in tasks:
            q = (f"On an NVIDIA B200, what limits a {t.operation} kernel at shape {t.shapes_text}, "
                 "and how would you restructure it?")
            a = teacher.generate([{"role": "user", "content": q}])
            rows.append({"messages": [{"role": "user", "content": q}, {"role": "assistant", "content": a}],
                         "_source": "qa", "task_id": t.task_id})
    write_jsonl(out, rows)
    return len(rows)
