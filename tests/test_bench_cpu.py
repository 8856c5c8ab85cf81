"""The bench's reference arm on the CPU (`bench.py --impl reference`): the JSON line the driver
reads, and the rule that only rank 0 works and prints under torchrun."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(extra_env=None, timeout=600):
    env = dict(os.environ)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                           "--warmup", "0"], cwd=ROOT, env=env, capture_output=True, text=True,
                          timeout=timeout)


def test_reference_arm_prints_one_contract_line():
    r = _run()
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 1
    assert d["steps"] == 1 and d["warmup"] == 0 and d["higher_is_better"] is True
    assert d["metric"] and d["unit"] == "tokens/s" and d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"]["workload"] and d["config"]["batch"] == 32
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"}, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_roofline_byte_counts_match_llama2_7b():
    """The algorithmic bytes behind `roofline.achieved`: every Llama-2-7B weight once per decode
    step (6.74 G linear parameters incl. the LM head = 13.48 GB in bf16) plus activations, and
    the live K/V rows of every sequence in every layer."""
    sys.path.insert(0, str(ROOT))
    import bench
    cfg = bench.LLAMA2_7B
    assert bench.layer_params(cfg) == 202_375_168
    weights = (32 * 202_375_168 + 32000 * 4096) * 2
    b = bench.decode_step_bytes(cfg, [1000] * 32)
    # Activations at batch 32 add about 1 % (inputs, outputs and residual reads of every GEMM).
    assert weights < b["gemm_decode"] < weights * 1.015
    assert b["gemm_decode"] == 13_353_828_352  # the figure the bench lines report
    kv = 32 * (32 * 1000) * 2 * 32 * 128 * 2        # layers x live rows x (K, V) x hkv x d x 2 B
    q_out = 32 * 2 * 32 * 32 * 128 * 2               # layers x (q, out) x B x hq x d x 2 B
    assert b["decode_attention"] == kv + q_out
    assert b["rmsnorm"] == (2 * 32 + 1) * (2 * 32 * 4096 * 2 + 4096 * 2)
