"""Message contract of the tool-using agent.

* Tool calls: Hermes ``<tool_call>{json}</tool_call>``, fenced ```json blocks,
  or OpenAI-style ``{"name", "arguments"}`` / ``{"function": {...}}``
  objects; string arguments holding JSON are decoded.
* Tool results: ``<tool_response>{"name", "content"}</tool_response>`` as a
  ``tool`` message.
* Reflection: a ``<reflection>...</reflection>`` block (or a ``Reflection:``
  paragraph) before the next call; counted for the tool-use shaping reward
  when it refers to the previous result.
* ``build_agent_system_prompt(tools, arch=..., phase=...)``: the kernel
  engineer prompt for the target architecture plus the tool list; the
  correctness phase and the optimisation phase differ only in their goal.
* ``episode_to_chat``: an episode's messages as a chat transcript for SFT
  (reasoning scratchpads dropped, tool results kept).

Reference behaviour: kore/agent/format.py:83-359.
"""
from __future__ import annotations

import json
import re
from typing import Dict, List, Optional

_HERMES = re.compile(r"<tool_call>\s*(\{.*?\})\s*</tool_call>", re.DOTALL)
_FENCE = re.compile(r"```(?:json)?\s*(\{.*?\})\s*```", re.DOTALL)
_REFLECT = re.compile(r"<reflection>(.*?)</reflection>|(?:^|\n)Reflection:\s*(.+?)(?:\n\n|$)", re.DOTALL | re.I)
_THINK = re.compile(r"<think>.*?</think>", re.DOTALL | re.I)

ARCHS = {
    "sm_100a": "NVIDIA B200 (sm_100a, Blackwell): 148 SMs, tcgen05 tensor cores with TMEM, TMA, "
               "thread-block clusters, 180 GB HBM3e",
    "sm_90a": "NVIDIA H100 (sm_90a, Hopper): 132 SMs, wgmma tensor cores, TMA, 80 GB HBM3",
}
PHASES = {
    "correctness": "Goal now: a CORRECT kernel. Build and test until every shape passes before optimising.",
    "optimize": "Goal now: make the correct kernel FASTER. Bench every change; revert when a change does not help.",
}


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


def render_tool_call(name: str, arguments: Dict) -> str:
    return "<tool_call>\n" + json.dumps({"name": name, "arguments": arguments}) + "\n</tool_call>"


def format_tool_result(name: str, result: Dict) -> str:
    return f"<tool_response>\n{json.dumps({'name': name, 'content': result}, default=str)}\n</tool_response>"


def parse_reflection(text: str) -> Optional[str]:
    for m in _REFLECT.finditer(_THINK.sub("", text or "")):
        body = (m.group(1) or m.group(2) or "").strip()
        if body:
            return body
    return None


def reflection_is_grounded(reflection: Optional[str], last_result: Optional[Dict]) -> bool:
    """A reflection counts when it mentions something the last tool result
    reported (an error, the correctness verdict, a timing or a speedup)."""
    if not reflection or not last_result:
        return False
    r = reflection.lower()
    keys = []
    if last_result.get("error"):
        keys += ["error", "compile", "fail"]
    if "correct" in last_result:
        keys += ["correct", "incorrect", "snr", "pass", "fail", "wrong"]
    if "wall_ms" in last_result or "speedup" in last_result:
        keys += ["ms", "faster", "slower", "speedup", "time", "bandwidth", "roofline"]
    return any(k in r for k in keys)


def build_agent_system_prompt(tools: List[Dict], arch: Optional[str] = None, phase: str = "correctness") -> str:
    from ..policy.format import SYSTEM_PROMPT
    target = ARCHS.get(arch or "sm_100a", ARCHS["sm_100a"])
    head = SYSTEM_PROMPT if (arch or "sm_100a") == "sm_100a" else SYSTEM_PROMPT.replace(
        SYSTEM_PROMPT.split("\n")[0], f"You are a GPU kernel engineer optimizing kernels for {target}.")
    spec = "\n".join(json.dumps(t) for t in tools)
    return (head + "\n" + PHASES.get(phase, PHASES["correctness"]) +
            "\nYou can call tools. Available tools (JSON schema):\n" + spec +
            "\nCall a tool with <tool_call>{\"name\": ..., \"arguments\": {...}}</tool_call>. "
            "Before each new call write a <reflection> on the previous tool result. "
            "Finish with `keep` on your best correct kernel.")


def episode_to_chat(messages: List[Dict], *, drop_think: bool = True) -> List[Dict]:
    out = []
    for m in messages:
        c = m.get("content", "")
        if drop_think and m.get("role") == "assistant":
            c = _THINK.sub("", c).strip()
        out.append({"role": m.get("role", "user"), "content": c})
    return out
