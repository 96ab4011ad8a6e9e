"""Data-factory generators on CPU (fake verifier env for the measured ones)."""
import zlib

from kore_b200.data import generators as G
from kore_b200.data.schemas import WinRecord
from kore_b200.reward.reward import Observation
from kore_b200.tasks.registry import get_task


class _Env:
    def __init__(self, task):
        self.task = task

    def step(self, src):
        h = zlib.crc32(src.encode())
        return Observation(compiled=True, validation_passed="broken" not in src, snr_db=60.0,
                           wall_ms=0.5 + (h % 5) / 10, baseline_ms=1.0)


def test_qa_is_grounded():
    tasks = [get_task("rmsnorm_bf16"), get_task("gemm_bf16")]
    wins = [WinRecord(task_id="gemm_bf16", trajectory=[], initial_wall_us=None, final_wall_us=None, speedup=1.5,
                      final_kernel="k1"),
            WinRecord(task_id="gemm_bf16", trajectory=[], initial_wall_us=None, final_wall_us=None, speedup=1.1,
                      final_kernel="k2")]
    qa = G.gen_qa(tasks, wins=wins, per_task=3)
    texts = [r["messages"][1]["content"] for r in qa]
    assert any("bound" in t for t in texts)
    assert any(t.startswith("A (1.50x") for t in texts)
    assert any(t == "148" for t in texts)


def test_reasoning_agentic_and_onpolicy():
    t = get_task("rmsnorm_bf16")
    env = _Env(t)
    rec = G.grounded_reasoning(t, t.seed_src, t.seed_src + "\n# faster", env)
    assert rec is None or "ANALYSIS:" in rec["messages"][1]["content"]
    ag = G.synth_agentic(t, [t.seed_src, t.seed_src + "\n# v2"], env)
    roles = [m["role"] for m in ag["messages"]]
    assert roles.count("tool") >= 4 and ag["final_kernel"]
    pol = lambda task: [f"FULL_KERNEL:\n```python\n{task.seed_src}\n```",
                        "FULL_KERNEL:\n```python\nbroken\n```", "no kernel here"]
    pairs = G.onpolicy_pairs([t], pol, lambda task: env)
    assert pairs and all(p["chosen"] != p["rejected"] for p in pairs)


def test_inductor_corpus_cpu():
    from kore_b200.tasks.ops_library import SPECS
    recs = G.synthetic_inductor_corpus([SPECS["gen_silu_mul_fp32"]], device="cpu", limit=1)
    assert len(recs) <= 1
    if recs:
        assert "operator: gen_silu_mul_fp32" in recs[0]["text"]


def test_breakers_cover_triton_and_cuda_and_have_hints():
    import random

    from kore_b200.data.factory import BREAKER_HINTS, BREAKERS, mutate
    assert set(BREAKERS) == set(BREAKER_HINTS)
    cu = ("__global__ void k(const float* x, float* y, int n) {\n  __shared__ float s[256];\n"
          "  int i = blockIdx.x * blockDim.x + threadIdx.x;\n  float acc = 0.f;\n  if (i < n) acc = x[i];\n"
          "  s[threadIdx.x] = acc;\n  __syncthreads();\n"
          "  acc += __shfl_xor_sync(0xffffffff, acc, off);\n  y[i] = acc;\n}\n")
    for name in ("drop_syncthreads", "cuda_bound_off_by_one", "wrong_thread_index", "wrong_shuffle_offset",
                 "cuda_half_accum"):
        out = BREAKERS[name](cu)
        assert out is not None and out != cu, name
    assert "if (i <= n)" in BREAKERS["cuda_bound_off_by_one"](cu)
    assert "(off + 1)" in BREAKERS["wrong_shuffle_offset"](cu)
    tri = "m = tl.sum(x, axis=1) / N\ny = acc * scale\n"
    assert BREAKERS["wrong_axis"](tri) == "m = tl.sum(x, axis=0) / N\ny = acc * scale\n"
    assert "/ N" not in BREAKERS["drop_normalization"](tri)
    assert "scale" not in BREAKERS["drop_scale"](tri)
    broken, op = mutate(cu, random.Random(0))
    assert broken != cu and op in BREAKERS
