"""SFT / midtrain / DPO trainers end to end on a tiny model (CPU, byte tokenizer)."""
import json
import math
import os

import pytest
import torch

from kore_b200.data.datasets import write_jsonl
from kore_b200.data.tokenizer import ByteTokenizer, render_chat
from kore_b200.models import qwen3_tiny
from kore_b200.parallel import dist as kd
from kore_b200.policy import dpo as dpo_mod
from kore_b200.policy.configs import DPOConfig, MidTrainConfig, SFTConfig
from kore_b200.policy.midtrain import pack_documents, train_midtrain
from kore_b200.policy.sft import train_sft


@pytest.fixture(autouse=True)
def _single():
    kd.shutdown()
    yield
    kd.shutdown()


def _cfg():
    return qwen3_tiny(vocab=512)


def test_render_chat_mask():
    tok = ByteTokenizer()
    ids, mask = render_chat(tok, [{"role": "user", "content": "hi"}, {"role": "assistant", "content": "yo"}])
    txt = tok.decode([i for i, m in zip(ids, mask) if m])
    assert txt == "yo<|im_end|>"


def test_sft_trains_and_checkpoints(tmp_path):
    rows = [{"messages": [{"role": "user", "content": f"q{i}"}, {"role": "assistant", "content": "a" * 20}],
             "_source": "repair" if i % 2 else "gen"} for i in range(8)]
    write_jsonl(tmp_path / "d.jsonl", rows)
    cfg = SFTConfig(model_id="tiny", dataset_path=str(tmp_path / "d.jsonl"), output_dir=str(tmp_path / "o"),
                    per_device_train_batch_size=2, gradient_accumulation_steps=1, num_train_epochs=1,
                    learning_rate=3e-3, max_seq_length=256, bf16=False, save_steps=2, logging_steps=1,
                    warmup_ratio=0.0, lr_scheduler_type="constant")
    out = train_sft(cfg, model_cfg=_cfg(), tokenizer=ByteTokenizer())
    h = out["history"]
    assert out["steps"] == 6 and h[-1] < h[0]          # 12 rows (repair x2) / 2 per step
    assert os.path.exists(tmp_path / "o" / "config.json")
    assert os.path.isdir(tmp_path / "o" / "checkpoint-4")
    # resume picks up the checkpoint instead of restarting
    out2 = train_sft(cfg, model_cfg=_cfg(), tokenizer=ByteTokenizer())
    assert len(out2["history"]) == 2


def test_midtrain_packing_and_train(tmp_path):
    tok = ByteTokenizer()
    wins = pack_documents(["x" * 50, "y" * 30], tok, 32)
    assert all(sum(len(d) for d in w) <= 32 for w in wins) and sum(len(d) for w in wins for d in w) == 82
    write_jsonl(tmp_path / "c.jsonl", [{"text": "hello world " * 10}] * 4)
    cfg = MidTrainConfig(model_id="tiny", corpus_path=str(tmp_path / "c.jsonl"), output_dir=str(tmp_path / "m"),
                         max_seq_length=64, per_device_train_batch_size=1, gradient_accumulation_steps=1,
                         learning_rate=3e-3, bf16=False, num_train_epochs=1, warmup_ratio=0.0,
                         lr_scheduler_type="constant")
    out = train_midtrain(cfg, model_cfg=_cfg(), tokenizer=tok)
    assert out["history"][-1] < out["history"][0]


def test_dpo_loss_derivatives():
    for lt in (["sigmoid"], ["ipo"], ["sigmoid", "sft"]):
        args = dict(rc=-5.0, rr=-6.0, nc=4, nr=5, beta=0.1, loss_types=lt, loss_weights=[1.0] * len(lt),
                    label_smoothing=0.1)
        l, dc, dr = dpo_mod.dpo_pair_loss(-4.0, -7.0, **args)
        e = 1e-5
        assert (dpo_mod.dpo_pair_loss(-4.0 + e, -7.0, **args)[0] - l) / e == pytest.approx(dc, rel=1e-3, abs=1e-7)
        assert (dpo_mod.dpo_pair_loss(-4.0, -7.0 + e, **args)[0] - l) / e == pytest.approx(dr, rel=1e-3, abs=1e-7)


def test_dpo_increases_margin(tmp_path):
    rows = [{"prompt": f"task {i}", "chosen": "good kernel " * 3, "rejected": "bad kernel " * 4} for i in range(4)]
    write_jsonl(tmp_path / "p.jsonl", rows)
    cfg = DPOConfig(model_id="tiny", dataset_path=str(tmp_path / "p.jsonl"), output_dir=str(tmp_path / "d"),
                    per_device_train_batch_size=2, gradient_accumulation_steps=1, num_train_epochs=2,
                    learning_rate=2e-3, bf16=False, max_length=256, beta=0.1, warmup_ratio=0.0,
                    lr_scheduler_type="constant")
    cfg.loss_type = ["sigmoid", "sft"]
    cfg.loss_weights = [1.0, 0.5]
    out = dpo_mod.train(cfg, model_cfg=_cfg(), tokenizer=ByteTokenizer())
    assert out["history"][-1] < out["history"][0]


def test_dpo_streamed_reference_and_micro_batches_match():
    """The frozen reference streamed layer by layer equals a resident one, and
    splitting the pairs into micro-batches gives the same gradient."""
    import torch

    from kore_b200.models import Qwen3Weights, qwen3_tiny
    from kore_b200.parallel.dist import get_context
    from kore_b200.policy.configs import DPOConfig
    from kore_b200.policy.dpo import DPOTrainer
    cfg = qwen3_tiny(vocab=512)
    g = torch.Generator().manual_seed(0)
    pairs = []
    for _ in range(2):
        p = torch.randint(0, 512, (9,), generator=g).tolist()
        pairs.append([(p + torch.randint(0, 512, (7,), generator=g).tolist(), 9),
                      (p + torch.randint(0, 512, (5,), generator=g).tolist(), 9)])
    grads = {}
    for place, mp in (("resident", 2), ("host", 1)):
        w = Qwen3Weights(cfg, device="cpu", dtype=torch.float32, seed=0)
        dt = DPOTrainer(DPOConfig(beta=0.1, learning_rate=1e-3, use_lora=False, bf16=False, ref_placement=place,
                                  micro_pairs=mp), get_context(), w)
        dt.tr.opt.step = lambda *a, **k: None
        dt.step(pairs)
        grads[place] = [x.clone() for x in dt.tr.eng.grads]
        assert dt.ref_placement == place
    for a, b in zip(grads["resident"], grads["host"]):
        assert torch.allclose(a, b, atol=1e-6, rtol=1e-4)
