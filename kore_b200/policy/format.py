"""Prompt / response contract of the kernel-writing policy (B200 target).

A response carries three sections, optionally preceded by a ``<think>``
scratchpad:

    ANALYSIS: what limits the current kernel (roofline, counters, feedback)
    PROPOSED_CHANGE: the one change this turn makes
    FULL_KERNEL:
    ```python
    <complete kernel module>
    ```

``parse_response`` is robust to missing headers and bare fenced blocks; the
scratchpad never leaks into the parsed sections. The multi-turn transcript
re-renders earlier turns without their reasoning (CoT masking) and appends
the verifier's feedback for each turn. Behavioural parity:
kore/policy/format.py:63-718 (system prompt retargeted to sm_100a).
"""
from __future__ import annotations

import re
from typing import Any, Dict, List, Optional

ANALYSIS, PROPOSED, FULL_KERNEL = "ANALYSIS", "PROPOSED_CHANGE", "FULL_KERNEL"
_THINK_RE = re.compile(r"<think\s*>(.*?)</think\s*>", re.DOTALL | re.IGNORECASE)
_FENCE = r"```(?:python|py|cuda|cpp|c\+\+)?\s*\n(.*?)```"

SYSTEM_PROMPT = """\
You are a GPU kernel engineer optimizing kernels for NVIDIA B200 (sm_100a, Blackwell):
148 SMs, 228 KB shared memory per SM (227 KB per block), 256 KB tensor memory (TMEM) per SM,
126 MB L2, 180 GB HBM3e at ~7.7 TB/s, 5th-generation tensor cores (tcgen05, bf16 2.25 PFLOP/s
dense, fp8 4.5), TMA bulk-tensor copies, thread-block clusters, 32-thread warps.

You receive a reference implementation, the current kernel and the verifier's feedback
(correctness SNR per shape, timings against the vendor baseline, roofline attainment and
hardware counters). Make ONE focused change per turn. The kernel must compute the result
itself: calling cuBLAS, cuDNN, CUTLASS library GEMMs, flashinfer, flash-attn or torch ops is
rejected as a reward hack, as are reading the environment, sleeping, spawning processes,
writing files, and printing verifier lines.

Answer in exactly this format:
ANALYSIS: <bottleneck analysis>
PROPOSED_CHANGE: <the change>
FULL_KERNEL:
```python
<the complete kernel module, defining the same entry points as the current kernel>
```
"""

OUTPUT_CONTRACT = (f"{ANALYSIS}: ...\n{PROPOSED}: ...\n{FULL_KERNEL}:\n```python\n...\n```")


def split_think(text: str):
    think = "\n".join(m.strip() for m in _THINK_RE.findall(text or ""))
    body = _THINK_RE.sub("", text or "")
    # an unclosed <think> swallows the rest of the response
    if "<think" in body.lower():
        i = body.lower().index("<think")
        think = (think + "\n" + body[i:]).strip()
        body = body[:i]
    return think, body


def _section(text: str, header: str, stops) -> str:
    m = re.search(rf"{header}\s*:?", text, flags=re.IGNORECASE)
    if not m:
        return ""
    start, end = m.end(), len(text)
    for s in stops:
        sm = re.search(rf"\n\s*{s}\s*:?", text[start:], flags=re.IGNORECASE)
        if sm:
            end = min(end, start + sm.start())
    return text[start:end]


def extract_kernel(text: str) -> str:
    _, body = split_think(text or "")
    fk = re.search(rf"{FULL_KERNEL}\s*:?", body, flags=re.IGNORECASE)
    scope = body[fk.end():] if fk else body
    m = re.search(_FENCE, scope, flags=re.DOTALL)
    if m:
        return m.group(1)
    if fk:
        return scope
    m = re.search(_FENCE, text or "", flags=re.DOTALL)
    return m.group(1) if m else ""


def parse_response(text: str) -> Dict[str, str]:
    think, body = split_think(text or "")
    return {"analysis": _section(body, ANALYSIS, (PROPOSED, FULL_KERNEL)).strip(),
            "proposed_change": _section(body, PROPOSED, (FULL_KERNEL,)).strip(),
            "kernel": extract_kernel(text or "").strip(),
            "think": think.strip()}


def wrap_full_kernel(source: str) -> str:
    return f"{FULL_KERNEL}:\n```python\n{source.rstrip()}\n```"


def format_assistant_turn(analysis: str, proposed_change: str, kernel: str, think: str = "") -> str:
    head = f"<think>\n{think}\n</think>\n" if think else ""
    return f"{head}{ANALYSIS}: {analysis}\n{PROPOSED}: {proposed_change}\n{wrap_full_kernel(kernel)}"


def summarize_cot(text: str, max_chars: int = 2000) -> str:
    """Keep head and tail of an over-long reasoning block."""
    text = text or ""
    if len(text) <= max_chars:
        return text
    marker = "\n...[cot summarized]...\n"
    budget = max(0, max_chars - len(marker))
    return text[: budget - budget // 2] + marker + text[len(text) - budget // 2:]


def normalize_assistant(content: str) -> str:
    """Re-render any response in the canonical contract (drops the scratchpad)."""
    p = parse_response(content)
    return format_assistant_turn(p["analysis"], p["proposed_change"], p["kernel"])


_KNOB_RE = re.compile(r"\b(BLOCK_[A-Z]+|num_warps|num_stages|GROUP_SIZE_M|TILE_[A-Z]+|STAGES)\s*[=:]\s*(\d+)")


def _knobs(src: str) -> Dict[str, int]:
    return {k: int(v) for k, v in _KNOB_RE.findall(src or "")}


def check_change_consistency(analysis: str, prev_kernel: str, new_kernel: str,
                             proposed_change: str = "") -> Dict[str, Any]:
    """Does the claimed change match the diff? Flags claims of changing tile /
    warp / stage knobs that did not change, and 'no change' claims with a diff."""
    claim = f"{analysis}\n{proposed_change}".lower()
    before, after = _knobs(prev_kernel), _knobs(new_kernel)
    changed = {k for k in set(before) | set(after) if before.get(k) != after.get(k)}
    claimed = {k for k in set(before) | set(after) if k.lower() in claim}
    identical = (prev_kernel or "").strip() == (new_kernel or "").strip()
    issues = []
    for k in sorted(claimed - changed):
        if k in before or k in after:
            issues.append(f"claims to change {k} but it is unchanged")
    if identical and proposed_change.strip():
        issues.append("proposes a change but the kernel is identical")
    return {"consistent": not issues, "issues": issues, "changed_knobs": sorted(changed)}


def _worst(d: dict):
    vals = [v for v in (d or {}).values() if v is not None]
    return min(vals) if vals else None


def build_turn_feedback(obs: Any, cfg: Any = None) -> str:
    """Verifier feedback text for the next turn."""
    if obs is None:
        return "No verifier result."
    if getattr(obs, "flagged_hack", False) or getattr(obs, "hack_reason", None):
        return f"REJECTED as a reward hack: {getattr(obs, 'hack_reason', '')}"
    if getattr(obs, "infra_error", False):
        return f"Infrastructure error (not your fault): {getattr(obs, 'error_text', '')}"
    if not getattr(obs, "compiled", False):
        return "Compile/runtime error:\n" + (getattr(obs, "error_text", "") or "")[-2000:]
    lines = []
    snrs = getattr(obs, "snr_by_shape", {}) or {}
    if snrs:
        lines.append("SNR per shape (dB): " + ", ".join(f"{k}={v:.1f}" for k, v in snrs.items()
                                                        if v is not None))
    if not getattr(obs, "validation_passed", False):
        lines.append("INCORRECT: output does not match the reference." +
                     (f" worst SNR {_worst(snrs):.1f} dB." if _worst(snrs) is not None else ""))
        if getattr(obs, "error_text", None):
            lines.append(obs.error_text[-1500:])
        return "\n".join(lines)
    walls = getattr(obs, "wall_by_shape", {}) or {}
    bases = getattr(obs, "baseline_by_shape", {}) or {}
    for k, w in walls.items():
        b = bases.get(k)
        lines.append(f"shape {k}: {w:.4f} ms" + (f" vs baseline {b:.4f} ms ({b / w:.2f}x)" if b else ""))
    if getattr(obs, "cv_pct", None) is not None:
        lines.append(f"timing CV {obs.cv_pct:.1f}%")
    return "CORRECT.\n" + "\n".join(lines)


def build_task_prompt(task: Any) -> str:
    ref = getattr(task, "reference_src", "") or ""
    seed = getattr(task, "seed_src", "") or ""
    shapes = getattr(task, "shapes_text", "") or ""
    return (f"Task: {getattr(task, 'task_id', '')} ({getattr(task, 'operation', '')}, "
            f"{getattr(task, 'dtype', '')}) on {getattr(task, 'gpu_target', 'sm_100a')}.\n"
            f"Shapes: {shapes}\n\nReference implementation:\n```python\n{ref}\n```\n\n"
            f"Current kernel:\n```python\n{seed}\n```\n\nRespond in the required format:\n{OUTPUT_CONTRACT}")


def build_transcript(task: Any, turns: List[dict], *, max_cot_chars: int = 0,
                     system: Optional[str] = None) -> List[Dict[str, str]]:
    """Chat messages for the next turn: system, task, then each earlier turn as
    an assistant message (reasoning dropped unless max_cot_chars > 0) followed
    by its verifier feedback as a user message."""
    msgs = [{"role": "system", "content": system or SYSTEM_PROMPT},
            {"role": "user", "content": build_task_prompt(task)}]
    for t in turns:
        if "response" in t and t["response"]:
            p = parse_response(t["response"])
        else:
            p = {"analysis": t.get("analysis", ""), "proposed_change": t.get("proposed_change", ""),
                 "kernel": t.get("kernel", ""), "think": t.get("think", "")}
        think = summarize_cot(p.get("think", ""), max_cot_chars) if max_cot_chars else ""
        msgs.append({"role": "assistant", "content": format_assistant_turn(
            p.get("analysis", ""), p.get("proposed_change", ""), p.get("kernel", ""), think)})
        fb = t.get("feedback") or (build_turn_feedback(t["obs"]) if t.get("obs") is not None else "")
        if fb:
            msgs.append({"role": "user", "content": f"Verifier feedback:\n{fb}"})
    return msgs
