"""The serving bench's request generators and KV checksum (bench_disagg.py), on the CPU:
BASELINE config 4's Poisson arrivals and length ranges, the closed-loop batches spread over the
decode groups, and the positional checksum the KV handoff checks bytes with."""
import pytest
import torch

import bench_disagg as bd
from hexgen2_b200.serving import Split


def test_poisson_requests_follow_config_4():
    reqs = bd._poisson(200, 2.0, seed=0, vocab=32000)
    arr = [r.arrival for r in reqs]
    assert arr[0] == 0.0 and all(b >= a for a, b in zip(arr, arr[1:]))
    mean_gap = arr[-1] / (len(arr) - 1)
    assert 0.4 < mean_gap < 0.6                      # 2 requests per second
    assert all(256 <= len(r.prompt) <= 2048 for r in reqs)
    assert all(64 <= r.max_new <= 512 for r in reqs)
    assert all(0 <= t < 32000 for r in reqs for t in r.prompt[:16])
    assert len({r.rid for r in reqs}) == 200
    again = bd._poisson(200, 2.0, seed=0, vocab=32000)   # seeded: the same workload every run
    assert [(r.arrival, r.prompt, r.max_new) for r in again] == [(r.arrival, r.prompt, r.max_new) for r in reqs]


@pytest.mark.parametrize("world,prefill", [(2, 1), (4, 1), (8, 2)])
def test_closed_loop_fills_every_decode_group_evenly(world, prefill):
    split = Split(world, prefill, 1)
    prompts = [[1] * n for n in (5, 9, 3)]
    reqs = bd._closed_loop(split, prompts, out_len=4, steps=2, rid0=100)
    assert len({r.rid for r in reqs}) == len(reqs) == 2 * len(prompts) * split.n_decode_groups
    for j in range(split.n_decode_groups):
        mine = [r for r in reqs if r.group == j]
        assert [r.index for r in mine] == list(range(2 * len(prompts)))
        assert [len(r.prompt) for r in mine] == [5, 9, 3] * 2


def test_positional_checksum_catches_changed_and_moved_words():
    buf = torch.arange(64, dtype=torch.int64).view(torch.uint8)
    ref = bd._positional_checksum(buf)
    assert bd._positional_checksum(buf.clone()) == ref
    swapped = buf.clone().view(torch.int64)
    swapped[[3, 4]] = swapped[[4, 3]]
    assert bd._positional_checksum(swapped.view(torch.uint8)) != ref   # same words, moved
    flipped = buf.clone()
    flipped[17] ^= 1
    assert bd._positional_checksum(flipped) != ref


def test_percentile_helper():
    assert bd._pct([], 0.5) is None
    assert bd._pct([3.0, 1.0, 2.0], 0.5) == 2.0
    assert bd._pct([1.0, 2.0, 3.0, 4.0], 0.9) == 4.0
