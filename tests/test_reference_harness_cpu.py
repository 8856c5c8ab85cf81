"""The reference's own harness on this package (CPU, hf-reference engine, seeded fixture): its
validate() (hexgen2/validate.py:11-50) and its two-rank prefill -> decode pilot
(hexgen2/run.py:65-218) with Engine, send_packet and recv_packet taken from hexgen2_b200, under
the assertions of the reference's runtime test (tests/test_runtime.py:14-40). Runs where the
reference checkout is present."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = Path(os.environ.get("HEXGEN2_REFERENCE", "/root/reference"))
pytestmark = pytest.mark.skipif(not (REF / "hexgen2" / "run.py").exists(),
                                reason="reference checkout not present")


def test_reference_validate_accepts_this_engine(fixture_dir):
    sys.path.insert(0, str(REF))
    try:
        import hexgen2.validate as validate_mod
        import hexgen2_b200 as hx
        saved = validate_mod.Engine
        validate_mod.Engine = hx.Engine
        try:
            result = validate_mod.validate(fixture_dir, "hf-reference", "cpu", "float32")
        finally:
            validate_mod.Engine = saved
    finally:
        sys.path.remove(str(REF))
    assert result["status"] == "passed"
    assert all(row["tokens_match"] for row in result["checks"])


def test_reference_pilot_runs_on_this_package(fixture_dir, tmp_path):
    out = tmp_path / "output"
    command = [sys.executable, "-m", "torch.distributed.run", "--standalone", "--nproc_per_node=2",
               "--local-addr", "127.0.0.1", str(ROOT / "tests" / "reference_pilot.py"), str(REF),
               "--model-dir", str(fixture_dir), "--trace", str(REF / "configs" / "tiny-trace.jsonl"),
               "--output", str(out), "--engine", "hf-reference", "--device", "cpu",
               "--dtype", "float32", "--check-colocated", "--profile-first"]
    result = subprocess.run(command, cwd=tmp_path, capture_output=True, text=True, timeout=300)
    assert result.returncode == 0, result.stderr[-3000:]
    records = [json.loads(s) for s in (out / "requests.jsonl").read_text().splitlines()]
    assert [r["output_tokens"] for r in records] == [1, 1, 4, 3]
    assert [r["warmup"] for r in records] == [True, False, False, False]
    assert all(r["colocated_matches"] and r["status"] == "success" for r in records)
    assert all(r["kv_packet_bytes"] > 0 for r in records)
    for rank in (0, 1):
        assert (out / f"rank-{rank}-trace.json.gz").is_file()
        events = [json.loads(s) for s in (out / f"rank-{rank}-events.jsonl").read_text().splitlines()]
        assert events[-1]["event"] == "complete"
    # As in the reference's test: a rerun into the same directory refuses to overwrite records.
    retry = subprocess.run(command, cwd=tmp_path, capture_output=True, text=True, timeout=300)
    assert retry.returncode != 0 and "Refusing to overwrite" in retry.stderr
