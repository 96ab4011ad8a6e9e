"""DPO on the GPU: a reference streamed from host memory (parked for the
update, its layer ring freed) and the one-GPU moment shuttle give the same
losses and parameters as a resident reference without the shuttle."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _pairs(vocab, n=4, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        p = torch.randint(0, vocab, (40,), generator=g).tolist()
        out.append([(p + torch.randint(0, vocab, (60,), generator=g).tolist(), 40),
                    (p + torch.randint(0, vocab, (45,), generator=g).tolist(), 40)])
    return out


def test_dpo_host_reference_and_shuttle_match_resident():
    from kore_b200.engine.smoke import smoke_config
    from kore_b200.models import Qwen3Weights
    from kore_b200.ops import check_device_error
    from kore_b200.parallel.dist import DistContext
    from kore_b200.policy.configs import DPOConfig
    from kore_b200.policy.dpo import DPOTrainer
    cfg = smoke_config()
    ctx = DistContext(device=torch.device("cuda"))
    pairs = _pairs(cfg.vocab_size)
    res = {}
    for place, shuttle in (("resident", "never"), ("host", "always")):
        w = Qwen3Weights(cfg, device="cuda", dtype=torch.bfloat16, seed=0)
        dt = DPOTrainer(DPOConfig(beta=0.1, learning_rate=1e-4, use_lora=False, bf16=True, ref_placement=place,
                                  micro_pairs=1), ctx, w, total_steps=4)
        dt.tr.moment_offload = shuttle
        losses = [dt.step(pairs) for _ in range(2)]
        assert dt.ref_placement == place
        if place == "host":
            assert dt._ref_stash.parked is False           # restored after the optimizer step
            assert dt.tr._shuttle is not None
        res[place] = (losses, [b.float().clone() for b in dt.tr.w.bufs])
    assert check_device_error() == 0
    assert all(abs(a - b) < 2e-3 for a, b in zip(res["resident"][0], res["host"][0])), res
    for a, b in zip(res["resident"][1], res["host"][1]):
        assert (a - b).abs().max() <= 4 * 1e-4 + 1e-6
