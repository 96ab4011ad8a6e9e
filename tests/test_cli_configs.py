"""Shipped configs, config schema strictness and the launcher (CPU)."""
import glob
import json

import pytest

from kore_b200 import cli
from kore_b200.policy import configs as C


def test_shipped_configs_parse():
    seen = set()
    for f in glob.glob("configs/*.json"):
        d = json.load(open(f))
        kind = f.split("/")[-1].split("_")[0]
        {"sft": lambda d: C.sft_config_from_dict(d)[0], "dpo": C.dpo_config_from_dict,
         "grpo": C.grpo_config_from_dict, "midtrain": C.midtrain_config_from_dict}[kind](d)
        seen.add(kind)
    assert seen == {"sft", "dpo", "grpo", "midtrain"}


def test_unknown_key_raises_and_extras_attach():
    with pytest.raises(TypeError):
        C.grpo_config_from_dict({"not_a_field": 1})
    d = C.dpo_config_from_dict({"loss_type": ["ipo", "sft"], "label_smoothing": 0.1})
    assert d.loss_type == ["ipo", "sft"] and d.label_smoothing == 0.1
    g = C.grpo_config_from_dict({"tasks": ["a"], "lora": {"r": 8}, "zero_stage": 2})
    assert g.zero_stage == 2


def test_sharding_plan_and_fsdp_kwargs():
    s = C.SFTConfig(distributed=True, use_lora=False)
    assert C.sharding_plan(s, 8)["zero"] == 3 and C.sharding_plan(s, 1)["zero"] == 0
    g = C.GRPOConfig(distributed=True)
    assert C.sharding_plan(g, 8)["zero"] == 2
    assert C.build_fsdp_kwargs(s)["fsdp_config"]["transformer_layer_cls_to_wrap"] == ["Qwen3DecoderLayer"]
    assert C.build_fsdp_kwargs(C.SFTConfig()) == {}
    assert C.build_deepspeed_config(g)["zero_optimization"]["stage"] == 3
    assert C.grpo_sharding_backend(g) == "fsdp"


def test_launch_dry_run(capsys):
    assert cli.main(["launch", "grpo", "configs/grpo_14b_full.json", "--gpus", "4", "--dry-run"]) == 0
    out = capsys.readouterr().out
    assert "--nproc-per-node=4" in out and "kore_b200.policy.grpo" in out and "127.0.0.1" in out
    with pytest.raises(SystemExit):
        cli.launch_command("nope", "x.json", 1)
