"""Shape augmentation: row-like dimension scaled and made non-aligned, byte
cap, and the environment failing a kernel that breaks on an augmented shape."""
import dataclasses
import json

from kore_b200.config import CONFIG
from kore_b200.env.kore_env import KoreEnv
from kore_b200.tasks.augment import augment_shapes, row_dim
from kore_b200.tasks.registry import get_task


def test_augmented_shapes():
    t = get_task("gen_silu_bf16")
    prim = t.shape("primary")
    k = row_dim(prim.dims)
    sh = augment_shapes(t)
    assert k in ("M", "T", "rows", "B", "S") and 2 <= len(sh) <= 3
    vals = [s.dims[k] for s in sh]
    assert any(v % 8 == 3 for v in vals) and all(v != prim.dims[k] for v in vals)
    for s in sh:                                       # only the row-like dimension changes
        assert {kk: vv for kk, vv in s.dims.items() if kk != k} == {kk: vv for kk, vv in prim.dims.items() if kk != k}
    assert augment_shapes(t, max_n=1) == sh[:1]
    assert augment_shapes(t, max_bytes=1.0) == []


def test_env_fails_kernel_on_augmented_shape(monkeypatch):
    t = get_task("gen_silu_bf16")
    cfg = dataclasses.replace(CONFIG, shape_augment=True, verifier_determinism_check=False)
    env = KoreEnv(t, cfg=cfg)
    calls = []

    def fake_exec(args, cwd, timeout=None):
        calls.append(args)
        if "--dims" in args:
            d = json.loads(args[args.index("--dims") + 1])
            if any(isinstance(v, int) and v % 8 == 3 for v in d.values()):
                return 0, "SNR: 4.00 dB\nallclose: False\nmax_diff: 3.0\n", False
        return 0, "SNR: 60.00 dB\nallclose: True\nmax_diff: 0.0001\n", False
    monkeypatch.setattr(env, "_exec", fake_exec)
    monkeypatch.setattr(env, "_bench", lambda *a, **k: None)
    obs = env.evaluate(t.seed_src)
    assert not obs.validation_passed and "augmented shape" in (obs.error_text or "")
    assert any("--dims" in c for c in calls)
    env2 = KoreEnv(t, cfg=dataclasses.replace(cfg, shape_augment=False))
    monkeypatch.setattr(env2, "_exec", fake_exec)
    monkeypatch.setattr(env2, "_bench", lambda *a, **k: None)
    assert env2.evaluate(t.seed_src + "\n").validation_passed


def test_data_scale_audit():
    from kore_b200.tasks.audit import audit
    r = audit()
    assert r.tasks >= 1334 and r.train + r.heldout == r.tasks and r.heldout >= 20
    assert sum(r.families.values()) == r.tasks and sum(r.dtypes.values()) == r.tasks
    assert r.with_roofline == r.tasks - r.external and r.augmented_shapes > r.tasks
    assert "tasks" in r.render()
