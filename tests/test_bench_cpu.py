"""The bench's reference arm runs on the host CPU alone and prints the
contract's JSON line (one line, the reference arm's keys)."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "e2e_1_5b", "--steps", "1",
                        "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "tokens/s"
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"] == "e2e_1_5b"
    # one step of this arm is one sampled forward of one sequence (one token)
    assert abs(d["ms_per_step"] - 1e3 / d["value"]) < 1e-6 * d["ms_per_step"]


def _bench():
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_roofline_arithmetic_and_traffic_lookup():
    b = _bench()
    peaks = {"hbm_gbs": 6500.0, "bf16_tflops": 1600.0, "src": "measured"}
    r = b.roofline_of({"bound": "hbm", "per_launch": 65e6, "kernel": "k"}, 0.01, peaks, "swiglu")
    assert r["bound"] == "hbm" and abs(r["achieved"] - 6500.0) < 1e-6 and abs(r["frac"] - 1.0) < 1e-9
    assert r["traffic"] == json.loads((ROOT / "profiles" / "traffic.json").read_text())["swiglu"]
    # 1 ms launches at the peaks: 1,600 TFLOP/s x 1 ms and 6,500 GB/s x 1 ms
    r = b.roofline_of({"bound": "tensor", "per_launch": 1.6e12, "kernel": "k", "hbm_bytes": 6.5e9}, 1.0, peaks, None)
    assert abs(r["frac"] - 1.0) < 1e-9 and abs(r["hbm_frac"] - 1.0) < 1e-9 and r["traffic"] is None
    assert b.roofline_of({"bound": "hbm", "per_launch": 1, "kernel": "k"}, None, peaks) is None


def test_e2e_dominant_kernel_choice():
    b = _bench()
    rows = [("nvjet_tst_256x256", 600, 190.0), ("fdl::block_attn_kernel<true>(fdl::AttnParams)", 868, 37.2),
            ("fdl::swiglu_kernel(fdl::SwigluArgs)", 896, 33.6)]
    assert b.e2e_dominant(rows) == ("block_attn_kernel", "block_attn_e2e")
    assert b.e2e_dominant(rows[:1] + rows[2:]) == ("swiglu_kernel", "swiglu")
    assert b.e2e_dominant(None) == ("swiglu_kernel", "swiglu")
    assert b.short_kernel_name("void fdl::gather_rmsnorm_kernel<__nv_bfloat16, 14>(fdl::NormArgs)") == \
        "fdl::gather_rmsnorm_kernel<__nv_bfloat16, 14>"


def test_kernel_suite_keys_have_committed_traffic():
    b = _bench()
    traffic = json.loads((ROOT / "profiles" / "traffic.json").read_text())
    for name, over, _ in b.KERNEL_SUITE:
        key = name if not over else f"{name}_b{over['attn_b']}_p{over['attn_p']}_sq{over['attn_sq']}"
        assert key in traffic, key
    assert "block_attn_e2e" in traffic
