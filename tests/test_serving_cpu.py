"""Host logic of the disaggregated serving pipeline (hexgen2_b200.serving), on the CPU: the
GPU-group split, request assignment and the staging ring's reservation protocol."""
import random

import pytest

from hexgen2_b200.serving import ALIGN, ByteRing, Request, Split, assign


@pytest.mark.parametrize("world,prefill,tp", [(2, 1, 1), (4, 1, 1), (8, 2, 1), (4, 2, 2), (8, 4, 4)])
def test_split_roles_and_pairing(world, prefill, tp):
    s = Split(world, prefill, tp)
    seen = {}
    for r in range(world):
        kind, g, t = s.role(r)
        ranks = s.prefill_ranks(g) if kind == "prefill" else s.decode_ranks(g)
        assert ranks[t] == r
        seen[r] = kind
    assert sum(k == "prefill" for k in seen.values()) == prefill
    # Every decode group has exactly one feeder; each decode rank pairs with the prefill rank of
    # the same TP index (equal-TP handoff, llama_disaggregate_with_tp_test.py:161, :170).
    fed = sorted(j for g in range(s.n_prefill_groups) for j in s.fed_by(g))
    assert fed == list(range(s.n_decode_groups))
    for j in range(s.n_decode_groups):
        for t in range(tp):
            p = s.prefill_ranks(s.feeder(j))[t]
            assert s.role(p) == ("prefill", s.feeder(j), t)


def test_split_for_throughput_and_rejects():
    assert (Split.for_throughput(2).prefill_gpus, Split.for_throughput(4).prefill_gpus,
            Split.for_throughput(8).prefill_gpus) == (1, 1, 2)
    assert Split.for_throughput(8, tp=4).prefill_gpus == 4
    for bad in [(2, 0, 1), (2, 2, 1), (4, 1, 2), (6, 2, 4)]:
        with pytest.raises(ValueError):
            Split(*bad)


def test_assign_round_robin_in_arrival_order():
    s = Split(8, 2, 1)  # 6 decode groups
    reqs = [Request(i, [1], 4, arrival=(7 * i) % 11) for i in range(30)]
    assign(reqs, s)
    order = sorted(reqs, key=lambda r: (r.arrival, r.rid))
    for n, r in enumerate(order):
        assert r.group == n % 6 and r.index == n // 6


def test_byte_ring_never_overwrites_unreleased_regions():
    """Random request sizes through a small ring: a reservation may only overlap regions the
    receiver has released, releases happen oldest first, and offsets are aligned."""
    rng = random.Random(0)
    size = 100 * ALIGN
    ring = ByteRing(size)
    released = []
    live = {}  # index -> (start, end) reserved and not yet released

    def wait(k):
        assert k == min(live), "release must be the oldest outstanding region"
        released.append(k)
        del live[k]

    for k in range(500):
        n = rng.randint(1, 40 * ALIGN)
        start = ring.reserve(k, n, wait)
        end = start + (n + ALIGN - 1) // ALIGN * ALIGN
        assert start % ALIGN == 0 and end <= size
        for s, e in live.values():
            assert e <= start or end <= s, "overlaps a region not yet released"
        live[k] = (start, end)
        # The receiver sometimes releases ahead of the sender's need.
        while live and rng.random() < 0.3:
            k0 = min(live)
            ring.live.popleft()
            released.append(k0)
            del live[k0]
    assert released == sorted(released)
    with pytest.raises(ValueError):
        ByteRing(ALIGN).reserve(0, 2 * ALIGN, wait)
