"""Multi-GPU self test of the data planes (run under torchrun, >= 2 GPUs).

    python -m torch.distributed.run --nproc-per-node N -m kore_b200.parallel.selftest

Checks: (1) three ZeRO-2 steps with NCCL collectives and with the fused
peer-memory optimizer give the same parameters (bf16 tolerance) and the
replicas stay bit-identical across ranks; (2) ZeRO-3 matches ZeRO-2 in loss
and final parameters, and ZeRO-3 with copy-engine peer gathers matches ZeRO-3
over NCCL; ZeRO-2 through the NVLink switch (multimem reduce / multicast
store) matches NCCL; (3) expert parallelism over NCCL all-to-all and over
the fused peer-memory dispatch/combine agree; (4) the tensor-parallel rollout
engine's sampled log-probs match an fp32 single-GPU reference forward that
scores the same tokens (teacher forcing); (5) a GRPO step runs with the TP
engine in the loop and its shard equals the updated weights after the sync.
Prints one JSON line per check from rank 0 and exits non-zero on failure.
"""
from __future__ import annotations

import json
import os
import sys
import time

import torch


def check_ep(ctx, g) -> bool:
    """Expert parallelism: three training steps over NCCL all-to-all, over the
    fused push dispatch and over the fused pull dispatch (the gate/up GEMM
    stages its receive rows from the peers) agree in loss and expert weights."""
    from ..engine.trainer import CausalLMTrainer
    from ..models import Qwen3Config
    from ..ops import check_device_error
    ok = True
    mcfg = Qwen3Config(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                       num_attention_heads=4, num_key_value_heads=2, head_dim=128, model_type="qwen3_moe",
                       num_experts=8 * ctx.world, num_experts_per_tok=4, moe_intermediate_size=256,
                       max_position_embeddings=2048)
    ids_m = torch.randint(0, mcfg.vocab_size, (ctx.world * 2, 256), generator=g)[ctx.rank * 2:(ctx.rank + 1) * 2].cuda()
    mres = {}
    for comm, disp in (("nccl", "pull"), ("fused", "push"), ("fused", "pull")):
        tr = CausalLMTrainer(mcfg, ctx, lr=1e-3, max_grad_norm=1.0, seed=0, comm=comm, master="fp32",
                             micro_tokens_hint=512, ep_dispatch=disp)
        losses = [tr.train_step_device(ids_m) for _ in range(3)]
        torch.cuda.synchronize()
        key = comm if comm == "nccl" else f"fused_{disp}"
        mres[key] = ([float(l) for l in losses], [b.float().clone() for b in tr.w.expert_bufs.values()])
        del tr
    err2 = check_device_error()
    for key in ("fused_push", "fused_pull"):
        mok = all(abs(a - b) < 2e-2 * max(1.0, abs(a)) for a, b in zip(mres["nccl"][0], mres[key][0]))
        for a, b in zip(mres["nccl"][1], mres[key][1]):
            mok = mok and torch.allclose(a, b, atol=2e-2, rtol=0)
        if ctx.is_main:
            print(json.dumps({"check": f"ep_{key}_vs_nccl", "world": ctx.world, "ok": mok and err2 == 0,
                              "loss_nccl": mres["nccl"][0], "loss_fused": mres[key][0], "device_error": err2}),
                  flush=True)
        ok = ok and mok
    return ok and err2 == 0


def main(argv=None):
    from ..engine.trainer import CausalLMTrainer
    from ..models import Qwen3Config
    from .dist import init_distributed

    ctx = init_distributed()
    if os.environ.get("KORE_SELFTEST_ONLY") == "ep":      # the expert-parallel check alone
        ok = check_ep(ctx, torch.Generator().manual_seed(123))
        torch.distributed.barrier()
        return 0 if ok else 1
    cfg = Qwen3Config(vocab_size=4096, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128, max_position_embeddings=2048)
    g = torch.Generator().manual_seed(123)
    ids_all = torch.randint(0, cfg.vocab_size, (ctx.world * 2, 256), generator=g)
    mine = ids_all[ctx.rank * 2:(ctx.rank + 1) * 2].cuda()
    res = {}
    for comm in ("nccl", "fused"):
        tr = CausalLMTrainer(cfg, ctx, lr=1e-3, max_grad_norm=1.0, seed=0, comm=comm, master="fp32")
        losses = [tr.train_step_device(mine) for _ in range(3)]
        torch.cuda.synchronize()
        res[comm] = ([float(l) for l in losses], [b.float().clone() for b in tr.w.bufs])
        del tr
    ok = True
    for a, b in zip(res["nccl"][1], res["fused"][1]):
        if not torch.allclose(a, b, atol=2e-2, rtol=0):   # bf16 params after 3 steps
            ok = False
    # replica consistency: checksum of the fused run on all ranks
    cs = torch.tensor([float(sum(b.double().sum() for b in res["fused"][1]))], device="cuda", dtype=torch.float64)
    lo, hi = cs.clone(), cs.clone()
    torch.distributed.all_reduce(lo, op=torch.distributed.ReduceOp.MIN)
    torch.distributed.all_reduce(hi, op=torch.distributed.ReduceOp.MAX)
    same = float(lo) == float(hi)
    from ..ops import check_device_error
    err = check_device_error()
    if ctx.is_main:
        print(json.dumps({"check": "zero2_fused_vs_nccl", "world": ctx.world, "ok": ok and same and err == 0,
                          "loss_nccl": res["nccl"][0], "loss_fused": res["fused"][0],
                          "replicas_identical": same, "device_error": err}), flush=True)
    # NVLink SHARP: gradients reduced in the switch, parameters multicast back
    from .nvls import NVLSUnavailable
    try:
        tr = CausalLMTrainer(cfg, ctx, lr=1e-3, max_grad_norm=1.0, seed=0, comm="nvls", master="fp32")
        ln = [float(tr.train_step_device(mine)) for _ in range(3)]
        torch.cuda.synchronize()
        nv_ok = all(abs(a - b) < 2e-2 * max(1.0, abs(a)) for a, b in zip(res["nccl"][0], ln))
        for a, b in zip(res["nccl"][1], tr.w.bufs):
            nv_ok = nv_ok and torch.allclose(a, b.float(), atol=2e-2, rtol=0)
        csn = torch.tensor([float(sum(b.double().sum() for b in tr.w.bufs))], device="cuda", dtype=torch.float64)
        lo2, hi2 = csn.clone(), csn.clone()
        torch.distributed.all_reduce(lo2, op=torch.distributed.ReduceOp.MIN)
        torch.distributed.all_reduce(hi2, op=torch.distributed.ReduceOp.MAX)
        errn = check_device_error()
        nv_ok = nv_ok and float(lo2) == float(hi2) and errn == 0
        del tr
        if ctx.is_main:
            print(json.dumps({"check": "zero2_nvls_vs_nccl", "world": ctx.world, "ok": nv_ok, "loss_nccl": res["nccl"][0],
                              "loss_nvls": ln, "replicas_identical": float(lo2) == float(hi2),
                              "device_error": errn}), flush=True)
        ok = ok and nv_ok
    except NVLSUnavailable as e:
        if ctx.is_main:
            print(json.dumps({"check": "zero2_nvls_vs_nccl", "world": ctx.world, "ok": True, "unavailable": str(e)}),
                  flush=True)
    # full sharding (ZeRO-3 layers: per-use gathers, per-micro-batch reduce-scatter on a comm stream)
    tr = CausalLMTrainer(cfg, ctx, lr=1e-3, max_grad_norm=1.0, seed=0, comm="nccl", master="fp32",
                         zero_stage=3, micro_batch_size=1)
    l3 = [float(tr.train_step_device(mine)) for _ in range(3)]
    full = tr.full_weights()
    torch.cuda.synchronize()
    z3ok = all(abs(a - b) < 2e-2 * max(1.0, abs(a)) for a, b in zip(res["nccl"][0], l3))
    for a, b in zip(res["nccl"][1], full.bufs):
        z3ok = z3ok and torch.allclose(a, b.float(), atol=2e-2, rtol=0)
    z3_params = [b.float().clone() for b in full.bufs]
    del tr, full
    if ctx.is_main:
        print(json.dumps({"check": "zero3_vs_zero2", "world": ctx.world, "ok": z3ok, "loss_zero2": res["nccl"][0],
                          "loss_zero3": l3}), flush=True)
    ok = ok and z3ok
    # ZeRO-3 with the layer gathers on the copy engines (peer reads of the symmetric heap)
    tr = CausalLMTrainer(cfg, ctx, lr=1e-3, max_grad_norm=1.0, seed=0, comm="fused", master="fp32",
                         zero_stage=3, micro_batch_size=1)
    l3f = [float(tr.train_step_device(mine)) for _ in range(3)]
    full = tr.full_weights()
    torch.cuda.synchronize()
    z3f = all(abs(a - b) < 1e-3 * max(1.0, abs(a)) for a, b in zip(l3, l3f))
    for a, b in zip(z3_params, full.bufs):
        z3f = z3f and torch.allclose(a, b.float(), atol=1e-3, rtol=0)
    errz = check_device_error()
    del tr, full
    if ctx.is_main:
        print(json.dumps({"check": "zero3_copy_engine_gather_vs_nccl", "world": ctx.world, "ok": z3f and errz == 0,
                          "loss_nccl": l3, "loss_ce_gather": l3f, "device_error": errz}), flush=True)
    ok = ok and z3f and errz == 0
    # expert parallelism: NCCL all-to-all vs fused peer-memory dispatch/combine
    mok = check_ep(ctx, g)
    err2 = 0
    ok = ok and mok
    # tensor-parallel rollout (AG->GEMM / GEMM->RS over peer memory) vs the 1-GPU engine
    from ..engine.rollout import GenRequest, RolloutEngine
    from ..models import Qwen3Weights
    from .tp import TPRolloutEngine
    tcfg = Qwen3Config(vocab_size=4096, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                       num_attention_heads=2 * ctx.world, num_key_value_heads=ctx.world, head_dim=128,
                       max_position_embeddings=2048)
    w = Qwen3Weights(tcfg, device="cuda", dtype=torch.bfloat16, seed=3)
    gp = torch.Generator().manual_seed(100 + ctx.rank)
    prompts = [torch.randint(0, tcfg.vocab_size, (n,), generator=gp).tolist() for n in (70, 33, 150)]
    tp = TPRolloutEngine(w, ctx, max_rows=1024, max_seqs=8, max_seq_len=512)
    toks, lps = tp.generate_static(prompts, 16, temperature=0.0)
    one = RolloutEngine(w, max_batch=8, page_size=64, num_pages=64, max_seq_len=512)
    ref_out = one.generate([GenRequest(p, 16, rid=i) for i, p in enumerate(prompts)], temperature=0.0)
    agree = sum(a == b for t, o in zip(toks, ref_out) for a, b in zip(t, o.tokens)) / max(1, sum(len(t) for t in toks))
    # teacher-forced: the fp32 reference scores the TP engine's own tokens (robust to greedy near-ties)
    from ..engine.qwen3_engine import Batch
    from ..models.reference_forward import forward_logprobs, leaf_buffers
    seqs = [torch.tensor(list(p) + t) for p, t in zip(prompts, toks)]
    b = Batch.from_sequences(seqs, device="cuda")
    with torch.no_grad():
        rlp, _ = forward_logprobs(w, [x.detach() for x in leaf_buffers(w)], b)
    lp_err, off = 0.0, 0
    for p, t, l in zip(prompts, toks, lps):
        ref_l = rlp[off + len(p) - 1: off + len(p) - 1 + len(t)].float().cpu().tolist()
        lp_err = max([lp_err] + [abs(a - c) for a, c in zip(l, ref_l)])
        off += len(p) + len(t)
    err3 = check_device_error()
    tok_ok = lp_err < 5e-2 and err3 == 0
    res_all = ctx.all_gather_object({"agree_greedy_1gpu": agree, "lp_err_teacher_forced": lp_err})
    if ctx.is_main:
        print(json.dumps({"check": "tp_rollout_vs_fp32_reference", "world": ctx.world,
                          "ok": all(r["lp_err_teacher_forced"] < 5e-2 for r in res_all), "ranks": res_all,
                          "device_error": err3}), flush=True)
    del tp, one
    # one GRPO step with the TP engine in the loop (multi-turn rollout, update,
    # in-place weight sync) next to the same step on the replicated engine
    from ..env.base import SyntheticRewardEnv
    from ..policy.configs import GRPOConfig
    from ..policy.grpo import GRPOTrainer
    from .tp import TPShard
    gstats = {}
    for mode in ("replica", "tp"):
        gw = Qwen3Weights(tcfg, device="cuda", dtype=torch.bfloat16, seed=4, pad_multiple=128 * ctx.world)
        gc = GRPOConfig(num_trajectories=4, num_turns=2, tasks_per_step=2, max_response_length=32,
                        max_prompt_length=1024, learning_rate=1e-4, temperature=1.0, dynamic_sampling=False,
                        starpo_s=False, total_steps=2, overlong_mask=False, rollout_parallel=mode)
        env = SyntheticRewardEnv(seed=0, prompt_len=96, feedback_len=8, vocab_size=tcfg.vocab_size)
        gt = GRPOTrainer(gc, weights=gw, env=env, ctx=ctx,
                         rollout_kwargs=dict(num_pages=256, page_size=64, max_seq_len=1024))
        st = gt.train_step(["a", "b"])
        st_ok = st["gen_tokens"] > 0 and bool(torch.isfinite(torch.tensor(st["loss"])))
        if mode == "tp":
            fresh = TPShard(gt.w, ctx.rank, ctx.world)
            st_ok = st_ok and all(torch.equal(a[k], b[k]) for a, b in zip(gt.tp.shard.layers, fresh.layers)
                                  for k in a)
        gstats[mode] = {"ok": st_ok, "gen_tokens": st["gen_tokens"], "loss": st["loss"],
                        "ms_rollout": st.get("ms_rollout"), "ms_sync": st.get("ms_sync")}
        del gt, gw
    err4 = check_device_error()
    gok = all(v["ok"] for v in gstats.values()) and err4 == 0
    gall = ctx.all_gather_object(gok)
    if ctx.is_main:
        print(json.dumps({"check": "grpo_tp_step", "world": ctx.world, "ok": all(gall), "steps": gstats,
                          "device_error": err4}), flush=True)
    torch.distributed.barrier()
    return 0 if (ok and same and err == 0 and mok and err2 == 0 and tok_ok and all(gall)) else 1


if __name__ == "__main__":
    sys.exit(main())
