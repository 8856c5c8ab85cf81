"""Launcher for the reference's two-rank pilot (hexgen2/run.py `main`) with this package's Engine
and transport in place of the reference's own (test infrastructure, started under
torch.distributed.run by tests/test_reference_harness_cpu.py).

    python -m torch.distributed.run --standalone --nproc_per_node=2 tests/reference_pilot.py \
        <HexGen-2 checkout> <hexgen2/run.py arguments...>
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, sys.argv.pop(1))

import hexgen2.run as run  # noqa: E402  (the reference's pilot, unchanged)

import hexgen2_b200 as hx  # noqa: E402

run.Engine = hx.Engine
run.send_packet, run.recv_packet = hx.send_packet, hx.recv_packet

if __name__ == "__main__":
    run.main()
