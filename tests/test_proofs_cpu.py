"""Smokes / proofs on CPU and the shared-node datagen-array helpers."""
import json

from kore_b200 import proofs
from kore_b200.campaign.nodes import array_manifest, manifest_shard, merge_shards, sbatch_array_script


def test_proofs_cpu():
    assert proofs.smoke_sft("cpu")["ok"]
    r = proofs.prove_ops()
    assert r["ok"], r
    assert proofs.verify_breadth(limit=60)["ok"]
    assert proofs.repro_grpo_step(world=2, port=29641)["ok"]
    assert proofs.smoke_env(device="cpu")["ok"]            # skipped without a GPU
    assert proofs.prove_value_cold_start(groups=120, holdout=30)["ok"]


def test_datagen_array(tmp_path):
    costs = {f"t{i}": float(i + 1) for i in range(10)}
    parts = array_manifest(costs, 3, str(tmp_path / "m.json"))
    assert sorted(sum(parts, [])) == sorted(costs)
    assert manifest_shard(str(tmp_path / "m.json"), 1) == parts[1]
    loads = [sum(costs[t] for t in p) for p in parts]
    assert max(loads) - min(loads) <= max(costs.values())
    sh = sbatch_array_script(str(tmp_path / "m.json"), "repair", str(tmp_path), shards=3, partition="gpu")
    assert "#SBATCH --array=0-2" in sh and "kore_b200.cli datagen repair" in sh
    a, b = tmp_path / "a.jsonl", tmp_path / "b.jsonl"
    a.write_text(json.dumps({"task_id": "x", "kernel": "k1"}) + "\n" + json.dumps({"task_id": "y", "kernel": "k"}) + "\n")
    b.write_text(json.dumps({"task_id": "x", "kernel": "k1"}) + "\n" + "not json\n")
    assert merge_shards([str(a), str(b), str(tmp_path / "missing")], str(tmp_path / "o.jsonl")) == 2
