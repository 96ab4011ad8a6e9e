"""General-capability retention suite: does kernel RL keep the base model's
other skills?

Six benchmarks, each a scorer over JSONL items that maps a model's response to
a score in [0, 1]:

* ``mmlu``      multiple choice; the first standalone choice letter in the answer.
* ``humaneval`` complete a Python function; the completion plus the item's
                asserts run in a sandboxed subprocess.
* ``livecodebench`` a stdin/stdout program; every test's stdout must match.
* ``ifeval``    verifiable formatting instructions (case, sentence / bullet /
                word counts, required / forbidden words, JSON keys, suffix).
* ``bfcl``      function calling; the first JSON object must name the expected
                function with matching arguments (numbers compared as numbers,
                strings case-insensitively).
* ``mtbench``   two-turn conversations scored by a judge callable; the default
                judge checks that each turn is answered and contains the
                reference key fact (no network judge offline).

Small smoke sets ship in ``kore_b200/eval/data`` (written for this package);
``load_bench(name, data_dir)`` reads a directory of full sets with the same
schema when one is provided. Generated code never runs in this process: each
program runs in a child Python with CPU-time and memory limits and a timeout.

Reference behaviour: kore/eval/retention.py:64-1109 (scorers, sandbox,
``run_retention_suite``).
"""
from __future__ import annotations

import json
import os
import re
import subprocess
import sys
import tempfile
from pathlib import Path
from typing import Callable, Dict, Iterable, List, Optional, Sequence

DATA = Path(__file__).resolve().parent / "data"
BENCHES = ("mmlu", "humaneval", "livecodebench", "ifeval", "bfcl", "mtbench")

Generate = Callable[[List[dict]], str]     # chat messages -> response text


def load_bench(name: str, data_dir: Optional[str] = None) -> List[dict]:
    d = Path(data_dir) if data_dir else DATA
    path = d / f"{name}.jsonl"
    if not path.exists():
        path = DATA / f"{name}.jsonl"
    with open(path) as f:
        return [json.loads(l) for l in f if l.strip() and not l.lstrip().startswith("#")]


# ----------------------------------------------------------------------------- sandbox
def run_python(code: str, stdin: str = "", timeout_s: float = 10.0, mem_mb: int = 1024) -> subprocess.CompletedProcess:
    """Run ``code`` in a child interpreter with resource limits (POSIX)."""
    with tempfile.TemporaryDirectory() as td:
        prog = Path(td) / "prog.py"
        prog.write_text(code)

        def limits():   # pragma: no cover - runs in the child
            import resource
            resource.setrlimit(resource.RLIMIT_AS, (mem_mb << 20, mem_mb << 20))
            cpu = int(timeout_s) + 1
            resource.setrlimit(resource.RLIMIT_CPU, (cpu, cpu))
        try:
            return subprocess.run([sys.executable, "-I", str(prog)], input=stdin, capture_output=True, text=True,
                                  timeout=timeout_s, cwd=td, preexec_fn=limits if os.name == "posix" else None)
        except subprocess.TimeoutExpired as e:
            return subprocess.CompletedProcess(e.cmd, -9, "", "timeout")


def extract_code(text: str) -> str:
    """The first fenced code block, else the text itself."""
    m = re.search(r"```(?:python|py)?\s*\n(.*?)```", text or "", re.DOTALL)
    return m.group(1) if m else (text or "")


def extract_json(text: str) -> Optional[dict]:
    s = text or ""
    for i, ch in enumerate(s):
        if ch != "{":
            continue
        depth = 0
        for j in range(i, len(s)):
            depth += {"{": 1, "}": -1}.get(s[j], 0)
            if depth == 0:
                try:
                    v = json.loads(s[i:j + 1])
                    return v if isinstance(v, dict) else None
                except json.JSONDecodeError:
                    break
    return None


# ----------------------------------------------------------------------------- scorers
class MMLU:
    name = "mmlu"

    @staticmethod
    def prompt(it):
        opts = "\n".join(f"{'ABCDEFGH'[i]}. {c}" for i, c in enumerate(it["choices"]))
        return [{"role": "user", "content": f"{it['question']}\n{opts}\nAnswer with the letter only."}]

    @staticmethod
    def score(it, resp: str) -> float:
        letters = "ABCDEFGH"[: len(it["choices"])]
        m = re.search(rf"\b([{letters}])\b", (resp or "").upper())
        return float(bool(m) and m.group(1) == str(it["answer"]).strip().upper())


class HumanEval:
    name = "humaneval"

    @staticmethod
    def prompt(it):
        return [{"role": "user", "content": "Complete this Python function. Reply with the full function in a "
                                            "```python``` block.\n\n" + it["prompt"]}]

    @staticmethod
    def score(it, resp: str) -> float:
        code = extract_code(resp)
        if f"def {it['entry_point']}" not in code:
            code = it["prompt"] + code
        r = run_python(code + "\n\n" + it["tests"])
        return float(r.returncode == 0)


class LiveCodeBench:
    name = "livecodebench"

    @staticmethod
    def prompt(it):
        return [{"role": "user", "content": it["question"] + "\nWrite a complete Python 3 program that reads stdin "
                                                             "and writes stdout, in a ```python``` block."}]

    @staticmethod
    def score(it, resp: str) -> float:
        code = extract_code(resp)
        for t in it["tests"]:
            r = run_python(code, stdin=t["input"])
            if r.returncode != 0 or r.stdout.strip() != str(t["output"]).strip():
                return 0.0
        return 1.0


def _sentences(t: str) -> List[str]:
    return [s for s in re.split(r"(?<=[.!?])\s+", t.strip()) if s]


_CHECKS: Dict[str, Callable[[dict, str], bool]] = {
    "lowercase": lambda s, r: r == r.lower() and any(c.isalpha() for c in r),
    "uppercase": lambda s, r: r == r.upper() and any(c.isalpha() for c in r),
    "sentence_count": lambda s, r: len(_sentences(r)) == s["n"],
    "bullet_count": lambda s, r: sum(1 for l in r.splitlines() if l.strip().startswith("- ")) == s["n"],
    "include_word": lambda s, r: s["word"].lower() in r.lower(),
    "exclude_word": lambda s, r: s["word"].lower() not in r.lower(),
    "max_words": lambda s, r: len(r.split()) <= s["n"],
    "json_keys": lambda s, r: (extract_json(r) or {"__": 0}).keys() == set(s["keys"]),
    "ends_with": lambda s, r: r.strip().endswith(s["text"]),
}


class IFEval:
    name = "ifeval"

    @staticmethod
    def prompt(it):
        return [{"role": "user", "content": it["prompt"]}]

    @staticmethod
    def score(it, resp: str) -> float:
        ins = it["instructions"]
        return sum(bool(_CHECKS[s["type"]](s, resp or "")) for s in ins) / max(1, len(ins))


def _same(a, b) -> bool:
    if isinstance(a, (int, float)) and not isinstance(a, bool):
        try:
            return abs(float(a) - float(b)) < 1e-9
        except (TypeError, ValueError):
            return False
    return str(a).strip().lower() == str(b).strip().lower()


class BFCL:
    name = "bfcl"

    @staticmethod
    def prompt(it):
        fns = json.dumps(it["functions"])
        return [{"role": "system", "content": f"You can call these functions: {fns}. Reply with one JSON object "
                                              '{"name": ..., "arguments": {...}}.'},
                {"role": "user", "content": it["question"]}]

    @staticmethod
    def score(it, resp: str) -> float:
        call = extract_json(resp)
        exp = it["expected"]
        if not call or call.get("name") != exp["name"]:
            return 0.0
        args = call.get("arguments") or {}
        return float(all(k in args and _same(v, args[k]) for k, v in exp["arguments"].items()))


def default_judge(question: str, answer: str, reference: str = "") -> float:
    """Offline judge: 0 for an empty answer, 1 when the reference key fact (if
    any) appears, 0.5 otherwise."""
    if not (answer or "").strip():
        return 0.0
    if not reference:
        return 1.0
    return 1.0 if reference.lower() in answer.lower() else 0.5


class MTBench:
    name = "mtbench"

    def __init__(self, judge: Callable[[str, str, str], float] = default_judge):
        self.judge = judge

    def run(self, it, generate: Generate) -> float:
        msgs: List[dict] = []
        scores = []
        for i, q in enumerate(it["turns"]):
            msgs.append({"role": "user", "content": q})
            a = generate(list(msgs))
            msgs.append({"role": "assistant", "content": a})
            ref = (it.get("reference") or [""] * len(it["turns"]))[i]
            scores.append(self.judge(q, a, ref))
        return sum(scores) / max(1, len(scores))


SCORERS = {c.name: c for c in (MMLU, HumanEval, LiveCodeBench, IFEval, BFCL)}


def score_bench(name: str, generate: Generate, items: Iterable[dict], judge=None) -> float:
    items = list(items)
    if not items:
        return 0.0
    if name == "mtbench":
        mt = MTBench(judge or default_judge)
        return sum(mt.run(it, generate) for it in items) / len(items)
    sc = SCORERS[name]
    return sum(sc.score(it, generate(sc.prompt(it))) for it in items) / len(items)


def run_retention_suite(generate: Generate, benches: Sequence[str] = BENCHES, *, data_dir: Optional[str] = None,
                        limit: Optional[int] = None, cache_path: Optional[str] = None, model_key: str = "model",
                        judge=None) -> Dict[str, float]:
    """Score every bench; results are cached per (model_key, bench)."""
    cache: Dict[str, float] = {}
    if cache_path and os.path.exists(cache_path):
        with open(cache_path) as f:
            cache = json.load(f)
    out: Dict[str, float] = {}
    for b in benches:
        key = f"{model_key}::{b}"
        if key not in cache:
            items = load_bench(b, data_dir)[: limit or None]
            cache[key] = score_bench(b, generate, items, judge)
        out[b] = cache[key]
    if cache_path:
        with open(cache_path, "w") as f:
            json.dump(cache, f, indent=1)
    return out


def engine_generate(tokenizer, engine, max_new_tokens: int = 256, eos_ids: Sequence[int] = ()) -> Generate:
    """A ``Generate`` on this package's rollout engine (greedy decoding)."""
    from ..data.tokenizer import render_chat
    from ..engine.rollout import GenRequest

    def gen(messages: List[dict]) -> str:
        ids, _ = render_chat(tokenizer, messages, add_generation_prompt=True)
        out = engine.generate([GenRequest(list(ids), max_new_tokens)], temperature=0.0, eos_ids=eos_ids)[0]
        return tokenizer.decode(out.tokens, skip_special_tokens=True)
    return gen
