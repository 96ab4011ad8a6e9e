"""Multi-process (gloo, world 2) runs of the trainers on CPU.

tiny Qwen3 policy (2 layers, hidden 256, 4 Q / 2 KV heads,
FFN 704, vocab 32000, fp32), one GRPO step on gloo world 2: 4 prompts of 64
uniform-random token ids (seed 0), group 4, 64-token completions, rewards
from the synthetic env, group-normalized advantages, clipped loss + KL to a
frozen copy. Plus: ZeRO-2 SFT on 2 ranks equals the 1-rank step."""
import os
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(fn, world, *args):
    port = _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_entry, args=(fn, r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in procs:
        r, v = q.get(timeout=600)
        out[r] = v
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.terminate()
    for r, v in out.items():
        if isinstance(v, str) and v.startswith("ERROR"):
            raise AssertionError(v)
    return out


def _entry(fn, rank, world, port, q, *args):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        from kore_b200.parallel import dist as kd
        ctx = kd.init_distributed(backend="gloo", timeout_s=300)
        q.put((rank, fn(ctx, *args)))
        kd.shutdown()
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, "ERROR " + traceback.format_exc()))


def _grpo_world2(ctx):
    from kore_b200.env.base import SyntheticRewardEnv
    from kore_b200.models import Qwen3Weights, qwen3_tiny
    from kore_b200.policy.configs import GRPOConfig
    from kore_b200.policy.grpo import GRPOTrainer
    torch.manual_seed(0)
    cfg = qwen3_tiny()
    w = Qwen3Weights(cfg, device="cpu", dtype=torch.float32, seed=0, pad_multiple=256)
    gc = GRPOConfig(num_trajectories=4, num_turns=1, tasks_per_step=4, max_response_length=64,
                    learning_rate=1e-4, temperature=1.0, ref_anchor_coef=1e-2, starpo_s=False,
                    dynamic_sampling=False, bf16=False, overlong_mask=False, clip_ratio_low=0.2,
                    clip_ratio_high=0.2)
    env = SyntheticRewardEnv(seed=0, prompt_len=64, feedback_len=4, vocab_size=cfg.vocab_size)
    tr = GRPOTrainer(gc, weights=w, env=env, ctx=ctx,
                     rollout_kwargs=dict(num_pages=64, page_size=32, max_seq_len=256))
    st = tr.train_step([0, 1, 2, 3])
    return {"samples": st["samples"], "checksum": float(sum(b.double().sum() for b in w.bufs)),
            "loss": st["loss"]}


def test_grpo_gloo_world2():
    out = _run(_grpo_world2, 2)
    assert out[0]["samples"] == 4 * 2 and out[1]["samples"] == 4 * 2   # 4 prompts x 4 / 2 ranks
    assert out[0]["checksum"] == pytest.approx(out[1]["checksum"], rel=0, abs=1e-6)  # replicas in sync


def _sft_zero(ctx):
    from kore_b200.engine.trainer import CausalLMTrainer
    from kore_b200.models import qwen3_tiny
    cfg = qwen3_tiny(vocab=512)
    tr = CausalLMTrainer(cfg, ctx, lr=1e-3, max_grad_norm=1.0, seed=0, dtype=torch.float32)
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, 512, (4, 32), generator=g)
    mine = ids[ctx.rank * 2:(ctx.rank + 1) * 2] if ctx.world > 1 else ids
    loss = tr.train_step(mine)
    return {"loss": loss, "w": [b[:1000].tolist() for b in tr.w.bufs]}


def test_zero2_sft_matches_single_rank():
    two = _run(_sft_zero, 2)
    one = _run(_sft_zero, 1)
    assert two[0]["loss"] == pytest.approx(one[0]["loss"], rel=1e-5)
    for a, b in zip(two[0]["w"], one[0]["w"]):
        assert torch.allclose(torch.tensor(a), torch.tensor(b), atol=1e-6)
    for a, b in zip(two[0]["w"], two[1]["w"]):
        assert a == b


def _moe_ep(ctx):
    from kore_b200.engine.trainer import CausalLMTrainer
    from kore_b200.models import Qwen3Weights
    from tests.test_moe_cpu import tiny_moe
    cfg = tiny_moe()
    full = Qwen3Weights(cfg, dtype=torch.float32, seed=5)
    ep = (ctx.rank, ctx.world) if ctx.world > 1 else None
    w = Qwen3Weights(cfg, dtype=torch.float32, init=False, pad_multiple=128 * ctx.world, ep=ep)
    for b in w.bufs:
        b.zero_()
    w.load_hf_state_dict(full.hf_state_dict())
    tr = CausalLMTrainer(cfg, ctx, lr=1e-3, max_grad_norm=1.0, seed=0, dtype=torch.float32, weights=w)
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, 256, (4, 24), generator=g)
    mine = ids[ctx.rank * 2:(ctx.rank + 1) * 2] if ctx.world > 1 else ids
    loss = tr.train_step(mine)
    return {"loss": loss, "sd": {k: v.flatten()[:64].tolist() for k, v in w.hf_state_dict().items()}}


def test_expert_parallel_matches_single_rank():
    two = _run(_moe_ep, 2)
    one = _run(_moe_ep, 1)
    assert two[0]["loss"] == pytest.approx(one[0]["loss"], rel=1e-5)
    for r in (0, 1):
        for k, v in two[r]["sd"].items():
            assert torch.allclose(torch.tensor(v), torch.tensor(one[0]["sd"][k]), atol=1e-6), k


def _sft_zero3(ctx):
    from kore_b200.engine.trainer import CausalLMTrainer
    from kore_b200.models import qwen3_tiny
    cfg = qwen3_tiny(vocab=512)
    tr = CausalLMTrainer(cfg, ctx, lr=1e-3, max_grad_norm=1.0, seed=0, dtype=torch.float32,
                         zero_stage=3 if ctx.world > 1 else 2, micro_batch_size=1)
    g = torch.Generator().manual_seed(7)
    out = []
    for step in range(2):
        ids = torch.randint(0, 512, (4, 32), generator=g)
        mine = ids[ctx.rank * 2:(ctx.rank + 1) * 2] if ctx.world > 1 else ids
        out.append(tr.train_step(mine))
    full = tr.full_weights()
    return {"loss": out, "w": [b[:1000].tolist() for b in full.bufs]}


def test_zero3_sft_matches_single_rank():
    """Full sharding (layer shards gathered per use, gradients reduce-scattered
    per micro-batch) gives the single-rank losses and weights."""
    two = _run(_sft_zero3, 2)
    one = _run(_sft_zero3, 1)
    for a, b in zip(two[0]["loss"], one[0]["loss"]):
        assert a == pytest.approx(b, rel=1e-5)
    for a, b in zip(two[0]["w"], one[0]["w"]):
        assert torch.allclose(torch.tensor(a), torch.tensor(b), atol=1e-5)
    for a, b in zip(two[0]["w"], two[1]["w"]):
        assert a == b


def _hb_worker(rank, world, path, die_rank, q):
    import torch.distributed as dist
    from kore_b200.parallel.health import Heartbeat, PeerFailure
    store = dist.FileStore(path, world)
    hb = Heartbeat(store, rank, world, timeout_s=2.0)
    done = 0
    try:
        for step in range(4):
            if step > 0:
                hb.wait_peers(step - 1)
            if rank == die_rank and step == 2:
                import os
                os._exit(0)                     # the rank vanishes between steps
            done = step
            hb.beat(step)
        q.put((rank, "ok", done))
    except PeerFailure as e:
        q.put((rank, "peer_failure", e.ranks))


def test_heartbeat_detects_dead_rank(tmp_path):
    """A rank that exits between steps is reported to every survivor on the
    host, within the heartbeat timeout, before their next step."""
    import multiprocessing as mp
    ctxm = mp.get_context("spawn")
    q = ctxm.Queue()
    world = 3
    path = str(tmp_path / "store")
    ps = [ctxm.Process(target=_hb_worker, args=(r, world, path, 1, q)) for r in range(world)]
    t0 = __import__("time").time()
    for p in ps:
        p.start()
    res = {}
    for _ in range(world - 1):
        r, kind, v = q.get(timeout=60)
        res[r] = (kind, v)
    for p in ps:
        p.join(timeout=30)
    assert res[0] == ("peer_failure", [1]) and res[2] == ("peer_failure", [1])
    assert __import__("time").time() - t0 < 45


def test_heartbeat_leave_and_classify():
    import torch.distributed as dist
    from kore_b200.parallel.health import Heartbeat, PeerFailure, classify_exception
    store = dist.HashStore()
    a, b = Heartbeat(store, 0, 2, timeout_s=0.2), Heartbeat(store, 1, 2, timeout_s=0.2)
    a.beat(0)
    b.beat(0)
    a.wait_peers(0)
    b.leave()
    with pytest.raises(PeerFailure):
        a.wait_peers(1)
    assert classify_exception(RuntimeError("CUDA out of memory")) == "infra"
    assert classify_exception(RuntimeError("NCCL error: unhandled system error")) == "infra"
    assert classify_exception(ValueError("bad shape")) == "program"


class _FakeKernelTask:
    def __init__(self, tid):
        self.task_id, self.operation, self.seed_src, self.dtype = tid, "rmsnorm", "def k(x): return x", "fp32"


class _FakeKernelEnv:
    """Stands in for KoreEnv: correctness and timing depend on a hash of the source."""

    def __init__(self, tid):
        self.task = _FakeKernelTask(tid)

    def step(self, src):
        import zlib

        from kore_b200.reward.reward import Observation
        h = zlib.crc32(src.encode())
        ok = h % 3 != 0
        return Observation(compiled=True, validation_passed=ok, snr_db=60.0 if ok else 5.0,
                           wall_ms=1.0 + (h % 7) / 10.0, baseline_ms=2.0)


class _FakeRolloutEnv:
    def __init__(self):
        self.envs = {}

    def _env(self, task):
        return self.envs.setdefault(task, _FakeKernelEnv(task))

    def prompt_messages(self, task):
        return [{"role": "user", "content": f"optimize {task}"}]


def _agentic_world2(ctx, out_dir):
    import kore_b200.agent.harness as H
    from kore_b200.data.tokenizer import ByteTokenizer
    from kore_b200.models import Qwen3Weights, qwen3_tiny
    from kore_b200.policy.configs import GRPOConfig
    from kore_b200.policy.grpo import GRPOTrainer
    calls = {"n": 0}

    def scripted(resp):   # the tiny random model cannot write tool calls: script them
        calls["n"] += 1
        return [{"name": "test", "arguments": {"source": f"def k(x): return x * {calls['n'] % 5}"}}]

    H.parse_tool_calls = scripted
    cfg = qwen3_tiny(vocab=512)
    w = Qwen3Weights(cfg, device="cpu", dtype=torch.float32, seed=0)
    gc = GRPOConfig(num_trajectories=4, num_turns=1, tasks_per_step=2, max_response_length=4,
                    max_prompt_length=512, learning_rate=1e-3, bf16=False, starpo_s=False, overlong_mask=False,
                    agentic=True, max_tool_turns=1, coevolve=True, use_search=True, search_every=1,
                    search_budget=4, coevolve_distill_path=os.path.join(out_dir, "wins.jsonl"),
                    dynamic_sampling=True, max_sampling_attempts=6, target_groups=2)
    tr = GRPOTrainer(gc, weights=w, env=_FakeRolloutEnv(), ctx=ctx, tokenizer=ByteTokenizer(512),
                     rollout_kwargs=dict(num_pages=256, page_size=16, max_seq_len=1024))
    st = tr.train_step(["t0", "t1"], max_new_tokens=4)
    picked = [e.desc.task_id for e in tr.curriculum.ctrl.archive.entries.values() if e.attempts]
    return {"samples": st["samples"], "groups": st["groups"], "picked": sorted(picked),
            "search": st.get("search"), "checksum": float(sum(b.double().sum() for b in w.bufs))}


def test_agentic_grpo_world2_with_curriculum_and_distill(tmp_path):
    """Agentic GRPO step on gloo world 2: tasks from the curriculum controller
    (same on both ranks), tool-using episodes, distributed dynamic sampling,
    rank-0 search-then-distill, identical replicas after the update."""
    out = _run(_agentic_world2, 2, str(tmp_path))
    assert out[0]["picked"] == out[1]["picked"] and out[0]["picked"]
    assert out[0]["groups"] >= 1 and out[0]["samples"] > 0
    assert out[0]["checksum"] == out[1]["checksum"]
    assert out[0]["search"] is not None and out[1]["search"] is None
    assert os.path.exists(tmp_path / "wins.jsonl")
