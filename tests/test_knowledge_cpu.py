"""B200 playbook injection and the experience ledger used during datagen."""
from kore_b200.data import knowledge as K
from kore_b200.policy.format import SYSTEM_PROMPT


def test_playbook_sections_and_live_prompt():
    secs = K.playbook_sections()
    for s in ("general", "gemm", "attention", "norm", "elementwise", "reduce", "moe", "quant", "pitfalls"):
        assert s in secs and secs[s].startswith("- ")
    assert K.sections_for("gemm_fused") == ["general", "gemm", "pitfalls"]
    assert K.sections_for("rmsnorm") == ["general", "norm", "pitfalls"]
    p = K.live_system_prompt(SYSTEM_PROMPT, operation="attention_decode")
    assert p.startswith(SYSTEM_PROMPT) and "[attention]" in p and "tcgen05" in p and "[gemm]" not in p
    short = K.live_system_prompt("base", operation="gemm", max_chars=200)
    assert len(short) <= len("base") + 60 + 200


def test_describe_change_names_schedule_edits():
    a = "BLOCK_M = 64\nnum_warps = 4\nacc += tl.dot(a, b)\n"
    b = "BLOCK_M = 128\nnum_warps = 8\nacc += tl.sum(a * b)\nx = tl.load(p, mask=m)\n"
    d = K.describe_change(a, b)
    assert "BLOCK_M 64 -> 128" in d and "num_warps 4 -> 8" in d and "removed tl.dot" in d and "added boundary masks" in d
    assert K.describe_change(a, a) == "a rewrite with the same schedule knobs"


def test_ledger_keeps_failures_dedups_and_caps():
    L = K.ExperienceLedger(max_items=3)
    a = "BLOCK_M = 64\n"
    assert not L.record("t", a, "BLOCK_M = 128\n", compiled=True, correct=True, parent_ms=1.0, child_ms=0.9)
    assert L.record("t", a, "BLOCK_M = 128\n", compiled=True, correct=True, parent_ms=1.0, child_ms=1.5)
    assert not L.record("t", a, "BLOCK_M = 128\n", compiled=True, correct=True, parent_ms=1.0, child_ms=1.6)
    assert L.record("t", a, "BLOCK_M = 16\n", compiled=False, correct=False, error="ptxas error : too much shared data")
    assert L.record("t", a, "BLOCK_M = 32\n", compiled=True, correct=False, error="SNR 3.1 dB below threshold")
    assert L.record("t", a, "BLOCK_M = 256\n", compiled=False, correct=False, error="error: out of resources")
    c = L.constraints("t")
    assert len(c) == 3 and "did not compile" in c[0] and "wrong results" in c[1]
    assert L.block("other") == ""


def test_generation_messages_do_not_touch_the_stored_turns():
    L = K.ExperienceLedger()
    L.record("t", "BLOCK = 64\n", "BLOCK = 8\n", compiled=False, correct=False, error="error: bad")
    stored = [{"role": "system", "content": SYSTEM_PROMPT}, {"role": "user", "content": "optimise"}]
    gen = K.generation_messages(stored, ledger=L, task_id="t")
    assert stored[0]["content"] == SYSTEM_PROMPT and stored[1]["content"] == "optimise"
    assert gen[0]["content"] != SYSTEM_PROMPT and "do not repeat" in gen[1]["content"]


def test_generators_store_the_canonical_prompt():
    from kore_b200.data.factory import generate_wins
    from kore_b200.tasks.registry import get_task

    class Obs:
        def __init__(self, ms, ok=True):
            self.compiled, self.validation_passed, self.wall_ms, self.snr_db = ok, ok, ms, 60.0
            self.error_text = None if ok else "error: x"
            self.speedup = None
            self.reward = 0.0

    seen = []

    class Teacher:
        def generate(self, msgs):
            seen.append(msgs)
            return "ANALYSIS: x\nPROPOSED_CHANGE: y\nFULL_KERNEL:\n```python\n" + t.seed_src.replace("def", "def", 1) + \
                "\n# v%d\n```" % len(seen)

    class Env:
        n = 0

        def step(self, src):
            Env.n += 1
            return Obs(1.0 / Env.n)

    t = get_task("gen_silu_bf16")
    recs = generate_wins([t], Teacher(), lambda task: Env(), turns=2, min_speedup=1.0)
    assert recs and recs[0].trajectory[0]["content"] == SYSTEM_PROMPT
    assert seen and "B200 optimisation notes" in seen[0][0]["content"]
