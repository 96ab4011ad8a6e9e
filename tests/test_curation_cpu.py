"""Dataset curation: hard negatives, repair->DPO, mixing, midtrain corpus,
DAgger relabel and sharded parallel datagen (with a fake verifier / launcher)."""
import json
import types

from kore_b200.data import curation
from kore_b200.data.schemas import RepairRecord, WinRecord
from kore_b200.tasks.registry import get_task

GOOD = """import torch
import triton
import triton.language as tl

@triton.jit
def _k(X, Y, N, BLOCK: tl.constexpr):
    m = tl.arange(0, BLOCK) < N
    x = tl.load(X + tl.arange(0, BLOCK), mask=m, other=0.0).to(tl.float32)
    y = tl.sum(x, 0)
    tl.store(Y, y)
"""


class FakeEnv:
    """Compiles everything except syntax slips; only the untouched source is correct."""

    def step(self, src):
        ok = src.strip() == GOOD.strip()
        return types.SimpleNamespace(compiled="):\n" in src or ok, validation_passed=ok, wall_ms=1.0 if ok else None)


def test_hard_negatives_are_compiling_but_wrong():
    t = get_task("rmsnorm_bf16")
    rows = curation.hard_negatives(t, GOOD, FakeEnv(), per_kernel=2, seed=1)
    assert rows and all(r["rejected"] != r["chosen"] for r in rows)
    assert len({r["negative"] for r in rows}) == len(rows)


def test_repair_to_dpo_and_mix_and_corpus(tmp_path):
    rec = RepairRecord("t", "snr_fail", "h", "err", [{"role": "user", "content": "broken"},
                                                    {"role": "assistant", "content": "fixed"}])
    pairs = curation.repair_to_dpo([rec])
    assert pairs[0]["chosen"] == "fixed" and "broken" in pairs[0]["rejected"]
    m = curation.mix({"a": [{"x": 1}], "b": [{"x": 2}]}, {"a": 3, "b": 1}, 40, seed=0)
    assert len(m) == 40 and sum(r["source"] == "a" for r in m) == 30
    docs = curation.midtrain_corpus([get_task("gemm_bf16")], [WinRecord("gemm_bf16", [], 2.0, 1.0, 2.0,
                                                                        final_kernel="k")],
                                    out_path=str(tmp_path / "c.jsonl"))
    assert len(docs) == 2 and all("text" in d for d in docs)


def test_dagger_and_parallel_datagen(tmp_path):
    from kore_b200.data.teacher import StubTeacher
    from kore_b200.policy.format import format_assistant_turn
    t = get_task("rmsnorm_bf16")
    teacher = StubTeacher(lambda m: format_assistant_turn("a", "b", GOOD))
    policy = StubTeacher(lambda m: "no kernel")
    pairs = curation.dagger_relabel([t], policy, teacher, lambda task: FakeEnv())
    assert len(pairs) == 1 and pairs[0]["rejected"] == "no kernel"
    (tmp_path / "repair-gpu0.jsonl").write_text(json.dumps({"task_id": "a"}) + "\n")
    launched = []
    shards = curation.parallel_datagen("repair", ["a", "b", "c", "d"], [0, 1], str(tmp_path),
                                       launcher=lambda cmd, env: launched.append((cmd, env["CUDA_VISIBLE_DEVICES"])))
    assert len(shards) == 2 and {e for _, e in launched} == {"0", "1"}
    tasks = ",".join(c[c.index("--tasks") + 1] for c, _ in launched)
    assert "a" not in tasks.split(",") and sorted(tasks.split(",")) == ["b", "c", "d"]


def test_general_replay_is_decontaminated_against_eval_prompts(tmp_path):
    import json

    from kore_b200.data.build_datasets import build_sft, eval_prompts
    ev = eval_prompts()
    assert len(ev) >= 5
    gen = tmp_path / "general.jsonl"
    rows = [{"messages": [{"role": "user", "content": ev[0]}, {"role": "assistant", "content": "x"}]},
            {"messages": [{"role": "user", "content": "Write a haiku about the ocean at dawn, please, "
                                                      "with a seasonal word."},
                          {"role": "assistant", "content": "waves"}]}]
    gen.write_text("\n".join(json.dumps(r) for r in rows) + "\n")
    out = tmp_path / "sft.jsonl"
    n = build_sft([], str(out), general=str(gen))
    kept = [json.loads(l) for l in out.read_text().splitlines()]
    assert n == 1 and "haiku" in kept[0]["messages"][0]["content"]
