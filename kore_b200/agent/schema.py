"""Agentic trajectory record (reference parity: kore/agent/schema.py:24)."""
from __future__ import annotations

from dataclasses import asdict, dataclass, field
from typing import List, Optional


@dataclass
class AgenticTrajectoryRecord:
    task_id: str
    messages: List[dict]
    tool_trace: List[dict] = field(default_factory=list)
    turn_rewards: List[float] = field(default_factory=list)
    turn_correct: List[bool] = field(default_factory=list)
    final_kernel: Optional[str] = None
    best_speedup: Optional[float] = None
    type: str = "agentic"

    def to_dict(self) -> dict:
        return asdict(self)
