"""Host-side pieces of bench.py that need no GPU: the committed ncu traffic lookup, the CPU
baseline (both dtypes of the reference's CPU path, on a tiny case), the clock summary, the
reference arm's non-zero ranks and the argument checks."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def test_traffic_comes_from_committed_profile():
    import bench
    lines = [ln.split() for ln in open(os.path.join(ROOT, "profiles", "traffic.txt")) if not ln.startswith("#")]
    table = {p[0]: float(p[1]) for p in lines if len(p) >= 2}
    assert bench._ncu_traffic("linear_gemm_kernel") == table["linear_gemm_kernel"]
    assert bench._ncu_traffic("act_quant_kernel") == table["act_quant_kernel"]
    assert bench._ncu_traffic("no_such_kernel") is None


@pytest.mark.parametrize("use_ref", [False, True])
def test_cpu_baseline_times_both_dtypes(monkeypatch, use_ref):
    import bench
    from krea2_svdquant_b200.quant import make_synthetic_state
    if use_ref and bench.reference_linear_fn() is None:
        pytest.skip("the reference is not installed in baseline/_ref")
    if not use_ref:
        monkeypatch.setattr(bench, "reference_linear_fn", lambda: None)
    m, k, n = 32, 128, 64
    monkeypatch.setattr(bench, "K", k)
    monkeypatch.setattr(bench, "OPS", 2 * m * n * k)
    x, st = make_synthetic_state(m, k, n, 8, 64, seed=0, device="cpu")
    tops, cores, sample, kind = bench.cpu_reference_tops(2, 1, x, st, budget_s=0.05)
    assert tops > 0 and cores >= 1
    assert "bf16" in sample and "fp32" in sample and "value = " in sample
    assert kind == ("reference" if use_ref else "port")


def test_reference_install_matches_port():
    """The reference's own svdquant_linear_sim (baseline/_ref) and the oracle's torch restatement
    that stands in for it give the same bf16 result on a small case."""
    import bench
    import torch
    from krea2_svdquant_b200.quant import make_synthetic_state
    from oracle.svdq_oracle import svdquant_linear_sim_torch
    ref = bench.reference_linear_fn()
    if ref is None:
        pytest.skip("the reference is not installed in baseline/_ref")
    sim, make_state = ref
    x, st = make_synthetic_state(32, 128, 64, 8, 64, seed=0, device="cpu")
    want = sim(x, make_state(st))
    got = svdquant_linear_sim_torch(x, st.smooth_scale, st.qweight, st.weight_scales, st.l1, st.l2, st.bias,
                                    group=64, k_in=128, k_pad=128)
    assert torch.equal(got, want)


def test_both_arms_share_config():
    import bench
    assert bench.bench_config(2) == bench.bench_config(2)
    assert {"workload", "M", "K", "N", "rank", "group", "l2", "parallelism"} <= set(bench.bench_config(1))


def test_clock_summary_ignores_idle_samples():
    import bench
    c = bench.ClockSampler(0)
    c.max_mhz = 1965
    c.samples = [300, 1500, 1510, 1490, 200]
    c.reasons = {"sw_power_cap"}
    s = c.summary()
    assert s["sm_mhz"] == 1500 and s["sm_max_mhz"] == 1965 and s["reasons"] == ["sw_power_cap"]


def test_reference_arm_nonzero_rank_exits_without_work():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2"],
                       env=env, capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0 and r.stdout.strip() == ""


def test_warmup_below_three_is_rejected():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--warmup", "2"],
                       capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode != 0 and "--warmup" in r.stderr


@pytest.mark.parametrize("flag", ["--only-block-linears", "--only-forward", "--only-small-batch",
                                  "--only-epilogues", "--offload", "--no-extra", "--graph"])
def test_documented_flags_exist(flag):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--help"],
                       capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0 and flag in r.stdout
