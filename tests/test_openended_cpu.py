"""Open-ended curriculum: typed grammar, construction gate, minting moves and
dedup, frontier scoring, controller determinism / feedback gathering /
checkpointing, held-out safety, competitor anchor."""
import math
import random

import pytest
import torch

from kore_b200.openended.archive import TaskArchive
from kore_b200.openended.competitor import competitor_regret
from kore_b200.openended.controller import CoevolutionController
from kore_b200.openended.grammar import Pipeline, lift, random_pipeline
from kore_b200.openended.minter import TaskMinter, gate_pipeline
from kore_b200.openended.proposer import Proposer
from kore_b200.openended.task_space import TaskDescriptor, TaskSpace


def test_typecheck():
    assert Pipeline(["matmul", "add_bias", "gelu"]).typecheck() is None
    assert "terminal" in Pipeline(["row_sum", "relu"]).typecheck()
    assert "unknown" in Pipeline(["attention"]).typecheck()
    rng = random.Random(0)
    for _ in range(50):
        assert random_pipeline(rng, rng.randint(1, 4)).typecheck() is None
    assert lift("gemm_bias_gelu").stages == ["matmul", "add_bias", "gelu"]


def test_gate_rejects_degenerates():
    assert gate_pipeline(Pipeline(["matmul", "silu", "rmsnorm"])) is None
    assert gate_pipeline(Pipeline(["softmax", "row_sum"])) == "constant output"   # rows of a softmax sum to 1
    assert gate_pipeline(Pipeline(["relu"]), family="paged_attention") == "held-out family"
    assert gate_pipeline(Pipeline(["row_max", "relu"])).startswith("ill-typed")


def test_reference_is_the_pipeline():
    p = Pipeline(["matmul", "add_residual", "rmsnorm"], width_out=32)
    x, w, r, s = p.build_sampler()({"M": 8, "N": 16}, 3, "cpu", torch.float32)
    want = x @ w.t() + r
    want = want * torch.rsqrt(want.pow(2).mean(-1, keepdim=True) + 1e-6) * s
    assert torch.allclose(p.build_reference()(x, w, r, s), want, atol=1e-5)
    f, b = p.cost(4096, 4096)
    assert f > 2 * 4096 * 4096 * 32 and p.intensity() > Pipeline(["relu"]).intensity()


def test_minter_registers_gated_unique_tasks():
    reg = {}
    m = TaskMinter(seed=3, registry=reg)
    ids = m.mint(6)
    assert len(ids) == 6 and len(set(ids)) == 6
    hashes = {(t.bhash, t.dtype) for t in m.minted}
    assert len(hashes) == 6
    for tid in ids:
        spec = reg[tid]
        ins = spec.make_inputs(spec.shapes["minimal"], 1, "cpu", torch.float32)
        y = spec.reference(*ins)
        assert torch.isfinite(y).all()
        assert torch.allclose(spec.baseline(*ins).float(), y, atol=1e-5)
        assert "NotImplementedError" in spec.seed_src
    again = TaskMinter(seed=3, registry={}).mint(6)
    assert again == ids                                   # deterministic for a seed


def test_frontier_scoring_zone_and_competitor():
    d = TaskDescriptor("t", "gemm", "gemm", "bf16", (("M", 4096), ("N", 4096), ("K", 4096)))
    a = TaskArchive()
    e = a.add(d)
    pr = Proposer()
    fresh = pr.score(e, [])
    for _ in range(80):
        a.record("t", 1.0)
    assert pr.score(a.entries["t"], []) == 0.0 < fresh     # mastered: outside the zone
    comp = Proposer(competitor={"t": 0.9, "u": float("nan")})
    e2 = TaskArchive().add(d)
    assert comp.score(e2, []) > Proposer().score(e2, [])
    assert comp._competitor("u") == 0.0
    assert competitor_regret({"t": 1.0}, {"t": 2.0, "z": -1}) == {"t": 0.5}


def test_controller_is_rank_deterministic_and_held_out_free():
    a, b = CoevolutionController(seed=5, batch=6), CoevolutionController(seed=5, batch=6)
    ia, ib = a.next_task_id(10), b.next_task_id(10)
    assert ia == ib and len(ia) == 10
    space = TaskSpace()
    assert all(d.family not in ("mla", "paged_attention") for d in space.items)

    class FakeCtx:
        world = 2

        def all_gather_object(self, obj):
            return [obj, [(t, 0.0, None) for t, _, _ in obj]]    # the other rank solved nothing
    c = CoevolutionController(seed=5, batch=6, ctx=FakeCtx())
    t = c.next_task_id(1)[0]
    c.record_batch([(t, 1.0, 1.5)])
    e = c.archive.entries[t]
    assert e.attempts == 1 and abs(e.succ_w - 0.5) < 1e-9 and e.best_speedup == 1.5
    st = c.state_dict()
    d = CoevolutionController(seed=5, batch=6)
    d.load_state_dict(st)
    assert d.next_task_id(3) == c.next_task_id(3)


def test_controller_mints_into_the_space():
    c = CoevolutionController(seed=1, batch=4, mint=True, mint_every=1, mint_batch=2)
    c.next_task_id(4)
    assert len(c.minted) == 2 and all(c.space.by_id(t) for t in c.minted)


def test_competitor_scores_mined_from_teacher_records(tmp_path):
    import json

    from kore_b200.openended import competitor as C
    p = tmp_path / "d.jsonl"
    rows = [{"type": "win", "task_id": "a", "speedup": 4.0},
            {"type": "win", "task_id": "b", "speedup": 0.9},
            {"type": "ranked_group", "task_id": "c", "parent_wall_us": 100.0,
             "candidates": [{"correct": True, "wall_us": 50.0, "snr_db": 60}, {"correct": False, "wall_us": 10.0}]},
            {"type": "win", "task_id": "d", "speedup": "nan?"}]
    p.write_text("\n".join(json.dumps(r) for r in rows) + "\nnot json\n")
    best = C.mine_teacher_speedups([str(p), str(tmp_path / "missing.jsonl")])
    assert best == {"a": 4.0, "b": 0.9, "c": 2.0}
    s = C.strength_scores(best, ref_percentile=1.0)
    assert s["a"] == 1.0 and s["b"] == 0.0 and 0.4 < s["c"] < 0.6
    r = C.build_competitor_scores([str(p)], ours={"a": 4.0, "c": 1.0})
    assert r["a"] == 0.0 and r["c"] == 0.5
    f = tmp_path / "s.json"
    C.save_scores(s, str(f))
    assert C.load_scores(str(f)) == pytest.approx(s) and C.load_scores(str(tmp_path / "x.json")) == {}
    assert C.summarize(s)["tasks"] == 3 and C.summarize({}) == {"tasks": 0}
