"""Disaggregated prefill/decode across GPU groups (multi-GPU bench path)."""
from __future__ import annotations


def run_bench_disaggregated(args):
    raise NotImplementedError("multi-GPU disaggregated bench is not built yet")
