"""Contract normalisation of training shards (SFT, DPO, raw records), kernel-
free and agentic rows untouched, idempotence, foreign-GPU marking."""
import json

from kore_b200.data import normalize as N
from kore_b200.policy.format import FULL_KERNEL, SYSTEM_PROMPT

OLD_SYS = "You are an expert Triton kernel engineer for AMD MI350X GPUs. Optimize the kernel."
RAW = "<think>hmm</think>\nCHANGE: tile\n```python\nimport triton\ndef k():\n    pass\n```"


def test_sft_row_is_rewritten_and_idempotent():
    row = {"messages": [{"role": "system", "content": OLD_SYS}, {"role": "user", "content": "task"},
                        {"role": "assistant", "content": RAW}]}
    out, ch = N.normalize_row(row)
    assert ch and out["messages"][0]["content"] == SYSTEM_PROMPT
    a = out["messages"][2]["content"]
    assert a.startswith("ANALYSIS:") and FULL_KERNEL in a and "import triton" in a and "<think>" not in a
    again, ch2 = N.normalize_row(out)
    assert not ch2 and again == out


def test_untouched_rows():
    chat = {"messages": [{"role": "system", "content": "You are a helpful assistant."},
                         {"role": "user", "content": "capital of France?"}, {"role": "assistant", "content": "Paris"}]}
    assert N.normalize_row(chat) == (chat, False)
    agent = {"messages": [{"role": "system", "content": OLD_SYS}, {"role": "assistant", "content": "<tool_call>{}"},
                          {"role": "tool", "content": "{}"}]}
    assert N.normalize_row(agent) == (agent, False)


def test_dpo_row_keeps_margin_and_wraps_kernels():
    row = {"prompt": [{"role": "system", "content": OLD_SYS}, {"role": "user", "content": "t"}],
           "chosen": RAW, "rejected": "```python\ndef k():\n    return 1\n```",
           "_provenance": {"margin": 0.3, "weight": 2.0}}
    out, ch = N.normalize_dpo_row(row)
    assert ch and out["chosen"].startswith(FULL_KERNEL) and out["rejected"].startswith(FULL_KERNEL)
    assert out["margin"] == 0.3 and out["weight"] == 2.0 and out["_provenance"] == row["_provenance"]
    assert out["prompt"][0]["content"] == SYSTEM_PROMPT


def test_file_in_place_with_backup_and_foreign_gpu(tmp_path):
    p = tmp_path / "s.jsonl"
    rows = [{"messages": [{"role": "system", "content": OLD_SYS}, {"role": "assistant", "content": RAW}]},
            {"type": "win", "task_id": "t", "trajectory": [], "speedup": 3.0, "gpu": "mi350x"}]
    p.write_text("\n".join(json.dumps(r) for r in rows) + "\nnot json\n")
    st = N.normalize_file(str(p), in_place=True, foreign_gpu=True)
    assert st == {"rows": 3, "changed": 2, "malformed": 1, "out": str(p)}
    assert (tmp_path / "s.jsonl.bak").exists()
    lines = p.read_text().splitlines()
    win = json.loads(lines[1])
    assert win["requires_reverify"] is True and win["gpu"] == "mi350x" and lines[2] == "not json"
