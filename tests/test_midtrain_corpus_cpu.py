"""Mid-training corpus: quality filters, chunking, held-out exclusion and
assembly from this repository's own sources (fast subset)."""
import json

from kore_b200.data import corpus_quality as Q
from kore_b200.data import midtrain_corpus as M


def test_code_and_doc_quality_reasons():
    good = "\n".join(f"__global__ void k{i}(float* x) {{ x[threadIdx.x] *= {i}.f; }}" for i in range(12))
    assert Q.code_quality_reason(good, "a.cu") is None
    assert Q.code_quality_reason("x = 1\n", "a.py") == "too_short"
    assert Q.code_quality_reason(good, "foo_pb2.py") == "generated_file"
    assert Q.code_quality_reason("a" * 3000 + "\n" + good, "a.cu") == "minified"
    assert Q.code_quality_reason("\n".join(["x = f(y)"] * 40), "a.py") == "repetitive"
    assert Q.code_quality_reason("ab\x00cd", "a.py") == "binary_or_empty"
    prose = " ".join(["The tensor memory accelerator moves tiles between global and shared memory."] * 8)
    assert Q.doc_quality_reason(prose, "a.md") is None
    assert Q.doc_quality_reason("# Title\n\nsee [x](http://a)\n", "a.md") == "too_little_prose"
    lic = "\n".join(["Copyright (c) 2024. Licensed under the Apache License. All rights reserved."] * 30) + "\nHello."
    assert Q.doc_quality_reason(lic, "LICENSE.md") in ("too_little_prose", "license_text")
    kept, why = Q.quality_filter([{"text": good, "path": "a.cu"}, {"text": "x=1", "path": "b.py"},
                                  {"text": "anything", "kind": "record"}])
    assert len(kept) == 2 and why == {"too_short": 1}


def test_chunking_respects_budget_and_lines():
    text = "".join(f"line {i}\n" for i in range(1000))
    parts = M.chunk_text(text, 500)
    assert all(len(p) <= 500 for p in parts) and "".join(parts) == text
    assert all(p.endswith("\n") for p in parts)


def test_heldout_mentions_and_assembly(tmp_path):
    assert M.mentions_heldout("uses genb_attn_prefill_sliding1k_h32kv8", ["genb_attn_prefill_sliding1k_h32kv8"])
    assert not M.mentions_heldout("nothing", ["short"])
    out = tmp_path / "c.jsonl"
    rep = M.build_midtrain_corpus(str(out), sources=["tasks", "repo_kernels", "docs"], max_docs=200)
    assert rep["docs"] > 0 and set(rep["by_source"]) <= {"tasks", "repo_kernels", "docs"}
    rows = [json.loads(l) for l in out.read_text().splitlines()]
    assert len(rows) == rep["docs"] and all(r["text"] for r in rows)
    from kore_b200.tasks.registry import split_tasks
    _, held = split_tasks()
    assert not any(r["path"] in held for r in rows if r["source"] == "tasks")
