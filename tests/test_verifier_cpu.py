"""Verifier: sm_100a occupancy model, Nsight Compute CSV parsers (long and
raw layouts), ptxas / nvcc report parsers, metric sets and derived metrics."""
import pytest

from kore_b200.verifier import occupancy as O
from kore_b200.verifier import pmc
from kore_b200.verifier.parsers import parse_ncu_long_csv, parse_ncu_raw_csv, parse_nvcc_diagnostics, \
    parse_ptxas_report


def test_occupancy_limits():
    # GEMM-like: 192 threads, 124 registers, ~225 KB of shared memory -> one block, smem-bound
    o = O.occupancy(192, 124, 225 * 1024, tmem_columns=512)
    assert o.blocks_per_sm == 1 and o.limiter in ("shared_memory", "tmem")
    # register-bound: 256 threads at 121 registers (rounded to 128) -> 65536 / (128*32*8) = 2
    o = O.occupancy(256, 121)
    assert o.blocks_per_sm == 2 and o.limiter == "registers" and o.warps_per_sm == 16
    # thread-bound: 1024 threads, few registers -> 2 blocks (64 warps)
    o = O.occupancy(1024, 16)
    assert o.blocks_per_sm == 2 and o.limiter == "threads" and o.occupancy == 1.0
    # block-count bound: tiny blocks
    o = O.occupancy(32, 16)
    assert o.blocks_per_sm == 32 and o.limiter == "blocks"
    # TMEM: 256 columns per block -> 2 blocks
    assert O.occupancy(128, 32, 0, tmem_columns=200).by_tmem == 2
    # invalid launches
    assert O.occupancy(2048).limiter == "invalid"
    assert O.occupancy(128, 300).limiter == "invalid"
    assert O.occupancy(128, 32, 230 * 1024).limiter == "invalid"


def test_waves_and_advice():
    w = O.waves(512, 1)
    assert w.full_waves == 3 and w.tail_blocks == 512 - 3 * 148
    assert w.tail_efficiency == pytest.approx(512 / (4 * 148))
    assert O.persistent_grid(2) == 296
    s = O.advise(O.occupancy(256, 121), grid=600)
    assert "limited by registers" in s and "waves" in s


LONG = ('==PROF== Connected\n'
        '"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size",'
        '"Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"\n'
        '"0","1","p","h","gemm_kernel","1","7","(192, 1, 1)","(148, 1, 1)","0","10.0","s",'
        '"gpu__time_duration.sum","usecond","208.70"\n'
        '"0","1","p","h","gemm_kernel","1","7","(192, 1, 1)","(148, 1, 1)","0","10.0","s",'
        '"dram__bytes_read.sum","Gbyte","1.25"\n'
        '"0","1","p","h","gemm_kernel","1","7","(192, 1, 1)","(148, 1, 1)","0","10.0","s",'
        '"sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active","%","94.70"\n'
        '"1","1","p","h","rmsnorm_bwd","1","7","(256, 1, 1)","(296, 1, 1)","0","10.0","s",'
        '"gpu__time_duration.sum","nsecond","93,888"\n'
        '"1","1","p","h","rmsnorm_bwd","1","7","(256, 1, 1)","(296, 1, 1)","0","10.0","s",'
        '"smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio","","6.37"\n'
        '"1","1","p","h","rmsnorm_bwd","1","7","(256, 1, 1)","(296, 1, 1)","0","10.0","s",'
        '"smsp__average_warps_issue_stalled_wait_per_issue_active.ratio","","2.61"\n'
        '"1","1","p","h","rmsnorm_bwd","1","7","(256, 1, 1)","(296, 1, 1)","0","10.0","s",'
        '"smsp__average_warps_issue_stalled_selected_per_issue_active.ratio","","1.00"\n')


def test_ncu_long_csv():
    ks = parse_ncu_long_csv(LONG)
    assert [k.kernel for k in ks] == ["gemm_kernel", "rmsnorm_bwd"]
    g, r = ks
    assert g.duration_ns == pytest.approx(208700.0) and g.dram_bytes == pytest.approx(1.25e9)
    assert g.threads_per_block == 192 and g.blocks == 148
    assert r.duration_ns == 93888.0
    assert r.top_stalls(2) == [("long_scoreboard", 6.37), ("wait", 2.61)]
    assert "tensor 94.7%" in g.summary()
    merged = pmc.parse_ncu_csv(LONG)                 # one dict, last kernel wins on shared names
    assert merged["gpu__time_duration.sum"] == 93888.0


RAW = ('"ID","Kernel Name","Block Size","Grid Size","gpu__time_duration.sum","dram__bytes_read.sum",'
       '"dram__bytes_write.sum","launch__registers_per_thread","lts__t_sector_hit_rate.pct"\n'
       '"","","","","usecond","Mbyte","Kbyte","register/thread","%"\n'
       '"0","gemm_kernel<256, 4, 0, 0>","(320, 1, 1)","(148, 1, 1)","529.82","300.5","512","124","61.5"\n')


def test_ncu_raw_csv_and_derived():
    (k,) = parse_ncu_raw_csv(RAW)
    assert k.kernel.startswith("gemm_kernel") and k.threads_per_block == 320
    assert k.metrics["dram__bytes_write.sum"] == 512e3 and k.metrics["launch__registers_per_thread"] == 124
    c = k.metrics
    assert pmc.dram_bytes(c) == pytest.approx(300.5e6 + 512e3)
    assert pmc.l2_hit_rate(c) == pytest.approx(0.615)
    assert pmc.achieved_bandwidth(c) == pytest.approx((300.5e6 + 512e3) / 529.82e-6)


def test_counter_variants_and_diagnosis():
    c = {"sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed": 44.7,
         "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed": 20.0,
         "sm__warps_active.avg.pct_of_peak_sustained_active": 30.0,
         "smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio": 6.4,
         "smsp__average_warps_issue_stalled_selected_per_issue_active.ratio": 1.0}
    assert pmc.tensor_busy_fraction(c) == pytest.approx(0.447)        # _active asked, _elapsed present
    d = pmc.diagnose(c)
    assert d.startswith("latency-bound") and "long_scoreboard" in d
    assert pmc.diagnose({"sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active": 90}).startswith("tensor")
    assert "memory-bound" in pmc.diagnose({"gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed": 88})
    assert "intensity" in pmc.diagnose({"dram__bytes_read.sum": 1e9}, flops=1e9)


def test_metric_sets_and_commands():
    assert pmc.metric_passes("standard") == [pmc.METRICS]
    g = pmc.metric_passes("grounding")
    assert len(g) == 4 and all(len(p) <= 17 for p in g)
    flat = [m for p in g for m in p]
    assert len(flat) == len(set(flat))                                  # passes share no metric
    with pytest.raises(KeyError):
        pmc.metric_passes("nope")
    cmd = pmc.ncu_command(["gpu__time_duration.sum"], ["python", "x.py"], kernel_regex="gemm", skip=2)
    assert cmd[:3] == ["ncu", "--clock-control", "none"] and "-c" in cmd and cmd[cmd.index("-c") + 1] == "1"
    assert "regex:gemm" in cmd and cmd[-2:] == ["python", "x.py"]


PTXAS = """ptxas info    : Compiling entry function '_ZN4kore18rmsnorm_bwd_kernelILi256ELi3EEEvPK13__nv_bfloat16' for 'sm_100a'
ptxas info    : Function properties for _ZN4kore18rmsnorm_bwd_kernelILi256ELi3EEEvPK13__nv_bfloat16
    0 bytes stack frame, 0 bytes spill stores, 0 bytes spill loads
ptxas info    : Used 121 registers, used 1 barriers, 32 bytes smem, 400 bytes cmem[0]
ptxas info    : Compiling entry function '_Z3bigv' for 'sm_100a'
ptxas info    : Function properties for _Z3bigv
    56 bytes stack frame, 108 bytes spill stores, 108 bytes spill loads
ptxas info    : Used 255 registers, used 1 barriers, 16 bytes smem, 380 bytes cmem[0], 8 bytes cmem[2]
"""


def test_ptxas_report_and_residency():
    r = parse_ptxas_report(PTXAS)
    a = r["_ZN4kore18rmsnorm_bwd_kernelILi256ELi3EEEvPK13__nv_bfloat16"]
    assert (a.registers, a.smem_bytes, a.barriers, a.cmem_bytes, a.has_spill) == (121, 32, 1, 400, False)
    assert a.residency(256).blocks_per_sm == 2
    b = r["_Z3bigv"]
    assert b.has_spill and b.stack_bytes == 56 and b.cmem_bytes == 388 and "SPILLS" in b.summary(128)
    assert pmc.parse_ptxas(PTXAS)["_Z3bigv"]["spill_loads"] == 108


def test_nvcc_diagnostics():
    text = ("kore_b200/csrc/x.cu(12): error: identifier \"foo\" is undefined\n"
            "kore_b200/csrc/x.cu(40): warning #177-D: variable \"y\" was declared but never referenced\n"
            "ptxas error   : Entry function '_Z1kv' uses too much shared data\n"
            "ptxas warning : Registers are spilled to local memory in function '_Z1kv'\n")
    errs, warns = parse_nvcc_diagnostics(text)
    assert [e["line"] for e in errs if e["file"]] == [12]
    assert any("too much shared data" in e["message"] for e in errs)
    assert len(warns) == 2 and warns[0]["line"] == 40


def test_collect_counters_runs_small_nvtx_captures(monkeypatch):
    import subprocess as sp
    from types import SimpleNamespace

    from kore_b200.tasks.registry import get_task
    calls = []

    def fake_run(cmd, **kw):
        calls.append(cmd)
        return SimpleNamespace(stdout=LONG, returncode=0)
    monkeypatch.setattr(pmc, "ncu_available", lambda: True)
    monkeypatch.setattr(sp, "run", fake_run)
    env = SimpleNamespace(task=get_task("gen_silu_bf16"), python="python", timeout=60, _env=lambda: {})
    c = pmc.collect_counters(env, "k.py", "/tmp", impl="baseline", metric_set="grounding")
    assert len(calls) == len(pmc.metric_passes("grounding"))
    for cmd in calls:
        assert cmd[:3] == ["ncu", "--clock-control", "none"] and "--nvtx-include" in cmd
        assert cmd[cmd.index("--nvtx-include") + 1] == "kore_profile/" and cmd[-2:] == ["--profile-run", "baseline"]
    assert c["gpu__time_duration.sum"] == 93888.0
