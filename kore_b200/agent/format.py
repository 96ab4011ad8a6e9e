"""Tool-call formats: Hermes ``<tool_call>{json}</tool_call>``, fenced
```json blocks, and OpenAI-style ``{"name", "arguments"}`` objects, plus the
agent system prompt (reference parity: kore/agent/format.py:83-359)."""
from __future__ import annotations

import json
import re
from typing import Dict, List, Optional

_HERMES = re.compile(r"<tool_call>\s*(\{.*?\})\s*</tool_call>", re.DOTALL)
_FENCE = re.compile(r"```(?:json)?\s*(\{.*?\})\s*```", re.DOTALL)


def parse_tool_calls(text: str) -> List[Dict]:
    calls = []
    for m in list(_HERMES.finditer(text or "")) or list(_FENCE.finditer(text or "")):
        try:
            d = json.loads(m.group(1))
        except json.JSONDecodeError:
            continue
        if "function" in d and isinstance(d["function"], dict):
            d = d["function"]
        name = d.get("name")
        args = d.get("arguments", d.get("parameters", {}))
        if isinstance(args, str):
            try:
                args = json.loads(args)
            except json.JSONDecodeError:
                args = {"raw": args}
        if name:
            calls.append({"name": name, "arguments": args or {}})
    return calls


def format_tool_result(name: str, result: Dict) -> str:
    return f"<tool_response>\n{json.dumps({'name': name, 'content': result})}\n</tool_response>"


def build_agent_system_prompt(tools: List[Dict]) -> str:
    from ..policy.format import SYSTEM_PROMPT
    spec = "\n".join(json.dumps(t) for t in tools)
    return (SYSTEM_PROMPT + "\nYou can call tools. Available tools (JSON schema):\n" + spec +
            "\nCall a tool with <tool_call>{\"name\": ..., \"arguments\": {...}}</tool_call>. "
            "Reflect on each tool result before the next call. Finish with `keep` on your best kernel.")
