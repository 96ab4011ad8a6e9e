"""Kernel environment logic that needs no GPU: registry/split, replay cache,
hack short-circuit, ncu / ptxas parsers, equivalence oracle on CPU ops."""
import torch

from kore_b200.env.kore_env import KoreEnv
from kore_b200.env.replay import ReplayCache
from kore_b200.reward.reward import Observation
from kore_b200.tasks.registry import all_tasks, get_task, split_tasks
from kore_b200.verifier.pmc import parse_ncu_csv, parse_ptxas
from kore_b200.verify.adversarial import coevolve_tests
from kore_b200.verify.equivalence import verify_equivalence


def test_registry_and_split():
    ids = [t.task_id for t in all_tasks()]
    assert "rmsnorm_bf16" in ids and "gemm_bf16" in ids and len(ids) >= 20
    tr, ho = split_tasks(seed=0)
    assert "quant_fp8_pertoken" in ho and "rmsnorm_bf16" in tr and not set(tr) & set(ho)
    t = get_task("rmsnorm_bf16")
    assert t.shape("primary").dims == {"M": 4096, "N": 5120} and "triton.jit" in t.seed_src


def test_hack_short_circuits_before_gpu():
    env = KoreEnv("gemm_bf16")
    obs = env.step("import torch\ndef gemm(a, b):\n    return torch.matmul(a, b.t())\n")
    assert obs.flagged_hack and "torch op" in obs.hack_reason


def test_replay_cache(tmp_path):
    p = tmp_path / "r.jsonl"
    c = ReplayCache(str(p))
    c.put("t", "src", Observation(compiled=True, snr_db=40.0))
    c.put("t", "bad", Observation(compiled=True, infra_error=True))
    c2 = ReplayCache(str(p))
    assert c2.get("t", "src").snr_db == 40.0 and c2.get("t", "bad") is None


def test_classify():
    env = KoreEnv("rmsnorm_bf16")
    assert env._classify(0, "SNR: 40\n", False) == "ok"
    assert env._classify(-9, "", True) == "infra"
    assert env._classify(3, "COMPILE_ERROR: SyntaxError", False) == "compile"
    assert env._classify(1, "RuntimeError: CUDA error: out of memory", False) == "infra"


def test_parsers():
    csv = ('"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Section Name",'
           '"Metric Name","Metric Unit","Metric Value"\n'
           '"0","1","p","h","k","1","7","s","dram__bytes_read.sum","Mbyte","134.5"\n'
           '"0","1","p","h","k","1","7","s","gpu__time_duration.sum","usecond","12.5"\n')
    d = parse_ncu_csv(csv)
    assert d["dram__bytes_read.sum"] == 134.5e6 and d["gpu__time_duration.sum"] == 12500.0
    rep = ("ptxas info    : Function properties for _Z3fooPf\n"
           "    0 bytes stack frame, 4 bytes spill stores, 8 bytes spill loads\n"
           "ptxas info    : Used 96 registers, used 1 barriers, 512 bytes smem\n")
    assert parse_ptxas(rep)["_Z3fooPf"] == {"spill_stores": 4, "spill_loads": 8, "registers": 96, "smem": 512}


def test_equivalence_oracle_and_coevolution():
    mk = lambda s: (torch.randn(64, 32, generator=torch.Generator().manual_seed(s)),)
    good = verify_equivalence(lambda x: torch.relu(x), lambda x: torch.relu(x), mk, family="unary")
    assert good.equivalent and good.false_accept_at_1pct < 1
    # wrong only on large inputs: random trials pass, the adversarial battery catches it
    bad = verify_equivalence(lambda x: torch.where(x.abs() > 10, 0 * x, torch.relu(x)),
                             lambda x: torch.relu(x), mk, family="unary")
    assert not bad.equivalent and bad.prongs["random"] and not bad.prongs["adversarial"]
    pop = coevolve_tests(mk, lambda x: torch.clamp(x, max=5.0), lambda x: x,
                         lambda a, b: float((a - b).abs().max()), population=6, generations=3)
    assert pop[0][1] > 0


def test_adversarial_hook_registry_and_replay(tmp_path):
    import torch
    from kore_b200.verify.adversarial_hook import AdversarialHook, AdversarialRegistry
    reg = AdversarialRegistry(str(tmp_path / "reg.json"))
    hook = AdversarialHook(reg, every=2, tol=1e-3, population=24, generations=3)
    make = lambda s: (torch.randn(64, 64, generator=torch.Generator().manual_seed(s)),)
    oracle = lambda x: torch.softmax(x.double(), -1).float()
    naive = lambda x: torch.exp(x) / torch.exp(x).sum(-1, keepdim=True)      # overflows on large inputs
    assert hook.on_accepted("softmax", "fp32", make, naive, oracle) == 0     # throttled: 1st of every 2
    added = hook.on_accepted("softmax", "fp32", make, naive, oracle)
    assert added > 0 and reg.genomes("softmax", "fp32")
    ok, _ = hook.replay("softmax", "fp32", make, naive, oracle)
    assert not ok
    ok, _ = hook.replay("softmax", "fp32", make, lambda x: torch.softmax(x, -1), oracle)
    assert ok
    assert AdversarialRegistry(str(tmp_path / "reg.json")).genomes("softmax", "fp32")
