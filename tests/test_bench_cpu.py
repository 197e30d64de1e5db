"""bench.py's reference arm (the oracle's restatement of the reference's CPU path, timed on the host
cores) on the CPU: one JSON line with the contract's keys, for a GEMM workload and the fused
element-wise workload in both evaluation precisions."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def reference_line(*extra):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0", "--cpu-seconds", "1", *extra], capture_output=True, text=True, timeout=300,
                       cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


@pytest.mark.parametrize("extra", [("--workload", "batched_gemm_bf16"), ("--workload", "gpt2_attention_bf16"),
                                   ("--workload", "fused_elementwise_f32"),
                                   ("--workload", "fused_elementwise_f32", "--expression", "gelu_chain",
                                    "--precision", "f32")])
def test_reference_arm_line(extra):
    d = reference_line(*extra)
    assert d["impl"] == "reference" and d["value"] > 0 and d["n_gpus"] == 1
    assert d["unit"] == d["cpu_baseline"]["unit"] == d["e2e"]["unit"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["config"]["workload"] == extra[1]
    assert d["ms_per_step_basis"].startswith("extrapolated")
    if extra[1] == "batched_gemm_bf16":  # the default workload carries the attention configuration too
        (att,) = d["secondary"]
        assert att["config"]["workload"] == "causal_attention_f16" and att["value"] > 0
        assert att["impl"] == "reference" and att["unit"] == "TFLOP/s"
    if "--precision" in extra:
        assert "gelu" in d["metric"] and "f32 evaluation" in d["metric"] and d["dtype"] == "f32"


def test_host_link_floor():
    """The e2e leg's copy floor: equal transfers take the concurrent rate throughout; for unequal
    ones the rest of the larger transfer moves at its rate alone once the smaller is done."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    bw = dict(h2d_gbs=50.0, d2h_gbs=60.0, bidir_h2d_gbs=40.0, bidir_d2h_gbs=40.0)
    assert b.host_link_floor_ms(40e9, 40e9, bw) == pytest.approx(1000.0)
    # 1 s together moves 40 GB each way; the remaining 20 GB of uploads take 0.4 s alone
    assert b.host_link_floor_ms(60e9, 40e9, bw) == pytest.approx(1400.0)
    assert b.host_link_floor_ms(40e9, 100e9, bw) == pytest.approx(2000.0)
    assert b.host_link_floor_ms(40e9, 0, bw) == pytest.approx(800.0)
