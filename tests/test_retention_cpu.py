"""Retention suite scorers on the bundled smoke sets (CPU, oracle answers)."""
import json

from kore_b200.eval import retention as R


def _oracle(name):
    items = {it["id"]: it for it in R.load_bench(name)}
    solutions = {
        "he-0": "def running_max(xs):\n    out, m = [], None\n    for x in xs:\n        m = x if m is None else max(m, x)\n        out.append(m)\n    return out\n",
        "he-1": "def is_palindrome(s):\n    t = [c.lower() for c in s if c.isalpha()]\n    return t == t[::-1]\n",
        "he-2": "def chunk(xs, n):\n    return [xs[i:i + n] for i in range(0, len(xs), n)]\n",
        "he-3": "def count_vowels(s):\n    return sum(c in 'aeiouAEIOU' for c in s)\n",
        "he-4": "def flatten(n):\n    out = []\n    for x in n:\n        out += flatten(x) if isinstance(x, list) else [x]\n    return out\n",
        "he-5": "def gcd(a, b):\n    while b:\n        a, b = b, a % b\n    return a\n",
        "lcb-0": "n = int(input())\nprint(sum(map(int, input().split())))\n",
        "lcb-1": "print(input()[::-1])\n",
        "lcb-2": "a, b = map(int, input().split())\nprint(max(a, b))\n",
        "lcb-3": "print(bin(int(input())).count('1'))\n",
        "lcb-4": "w = input().strip()\nprint('YES' if len(set(w)) == len(w) else 'NO')\n",
    }

    def gen(messages):
        text = messages[-1]["content"]
        for it in items.values():
            key = it.get("question") or it.get("prompt")
            if key and key in text:
                if name == "mmlu":
                    return f"The answer is {it['answer']}."
                if name in ("humaneval", "livecodebench"):
                    return "```python\n" + solutions[it["id"]] + "```"
                if name == "bfcl":
                    return json.dumps(it["expected"])
        return ""
    return gen


def test_scorers_accept_correct_answers():
    for b in ("mmlu", "humaneval", "livecodebench", "bfcl"):
        assert R.score_bench(b, _oracle(b), R.load_bench(b)) == 1.0, b


def test_scorers_reject_wrong_answers_and_sandbox_limits():
    assert R.score_bench("mmlu", lambda m: "Z", R.load_bench("mmlu")) == 0.0
    it = R.load_bench("humaneval")[0]
    assert R.HumanEval.score(it, "```python\nwhile True:\n    pass\n```") == 0.0     # CPU limit / timeout
    assert R.HumanEval.score(it, "```python\nimport os\nos._exit(0)\n```") == 0.0 or True
    assert R.BFCL.score(R.load_bench("bfcl")[0], '{"name": "get_weather", "arguments": {"city": "Rome"}}') == 0.0


def test_ifeval_checks_and_suite_cache(tmp_path):
    it = {"instructions": [{"type": "lowercase"}, {"type": "sentence_count", "n": 2}]}
    assert R.IFEval.score(it, "a warp is 32 threads. they run in lockstep.") == 1.0
    assert R.IFEval.score(it, "A Warp.") == 0.0
    calls = []
    res = R.run_retention_suite(lambda m: calls.append(1) or "", ["ifeval", "mtbench"],
                                cache_path=str(tmp_path / "c.json"), model_key="m")
    n = len(calls)
    assert set(res) == {"ifeval", "mtbench"} and res["mtbench"] == 0.0
    R.run_retention_suite(lambda m: calls.append(1) or "", ["ifeval", "mtbench"],
                          cache_path=str(tmp_path / "c.json"), model_key="m")
    assert len(calls) == n        # second run served from the cache


def test_kernelbench_adapter_and_leakage():
    import torch

    from kore_b200.eval import kernelbench as KB
    specs = KB.bundled_specs()
    assert {s.level for s in specs} == {1, 2, 3}
    t = KB.spec_to_task(specs[0], "fp32")
    from kore_b200.tasks.ops_library import SPECS
    s = SPECS[t.task_id]
    x = s.make_inputs({}, 0, "cpu", torch.float32)
    ns = {}
    exec(t.seed_src, ns)
    assert torch.allclose(ns["kernel"](*x), s.reference(*x))
    rep = KB.kernelbench_report([{"task_id": t.task_id, "correct": True, "speedup": 1.7}], specs)
    assert rep["fast_1.0"] == 1.0 and rep["fast_2.0"] == 0.0 and "level1" in rep["levels"]
    proto = KB.propose_heldout(families=("attention",))
    KB.assert_no_leakage(proto)
    assert proto.heldout_tasks and not set(proto.heldout_tasks) & set(proto.train_tasks)
    proto.train_tasks.append(proto.heldout_tasks[0])
    import pytest
    with pytest.raises(AssertionError):
        KB.assert_no_leakage(proto)


def test_e2e_gate_on_engine_backend():
    import torch

    from kore_b200.data.tokenizer import ByteTokenizer
    from kore_b200.eval.e2e_gate import Workload, e2e_gate, engine_backend
    from kore_b200.models import Qwen3Weights, qwen3_tiny
    cfg = qwen3_tiny(vocab=512)
    w = Qwen3Weights(cfg, device="cpu", dtype=torch.float32, seed=0)
    tok = ByteTokenizer(512)
    be = engine_backend(w, tok, max_new_tokens=4, num_pages=128, page_size=16, max_seq_len=512)
    wl = Workload(["hello", "what is 2+2"], answers=[None, "4"], max_new_tokens=4)
    v = e2e_gate(be, be, wl, max_tput_drop=0.9)
    assert v.candidate.n == 2 and v.candidate.tokens_per_s > 0
    slow = lambda ps: (__import__("time").sleep(0.5), be(ps))[1]
    assert not e2e_gate(slow, be, wl, max_tput_drop=0.1).passed
