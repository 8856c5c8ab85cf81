"""The tensor-parallel greedy token (GPTLMHeadModel.next_tokens): each rank's (value, index) of
its vocabulary slice packed into one int64 key, one all-reduce(MAX), and the winner equals
torch.argmax over the gathered logits — ties to the lowest index, negative maxima, -0.0 against
+0.0 — on 2 and 4 Gloo ranks."""
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hexgen2_b200.gpt import argmax_keys, key_index

V, B = 32000, 8


def _logits(dtype):
    g = torch.Generator().manual_seed(11)
    x = torch.randn(B, V, generator=g)
    x[1] = 0.5                                   # every index ties: index 0 wins
    x[2, 100] = x[2, V - 1] = 9.0                # tie across the first and the last slice
    x[3] = -torch.rand(V, generator=g) - 1.0     # all negative
    x[4] = -1.0                                  # max 0.0 on the last slice, -0.0 earlier
    x[4, 5] = -0.0
    x[4, V - 3] = 0.0
    x[5, V // 2] = float("inf")
    return x.to(dtype)


def _worker(rank, world, rendezvous, dtype_name):
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            init_method=Path(rendezvous).as_uri(), timeout=timedelta(seconds=30))
    try:
        logits = _logits(getattr(torch, dtype_name))
        vloc = V // world
        local = logits[:, rank * vloc:(rank + 1) * vloc]
        idx = local.float().argmax(-1)
        val = local.gather(1, idx.view(B, 1)).view(B)
        key = argmax_keys(val, idx + rank * vloc)
        dist.all_reduce(key, op=dist.ReduceOp.MAX)
        got = key_index(key)
        want = logits.float().argmax(-1)
        assert torch.equal(got, want), (got.tolist(), want.tolist())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("dtype_name", ["float32", "bfloat16"])
def test_tp_argmax_keys_equal_gathered_argmax(tmp_path, world, dtype_name):
    mp.spawn(_worker, args=(world, str(tmp_path / "rdzv"), dtype_name), nprocs=world, join=True)


def test_keys_order_values_then_lowest_index():
    vals = torch.tensor([-2.0, -0.0, 0.0, 1e-30, 3.0, 3.0])
    idx = torch.tensor([7, 1, 9, 4, 6, 2])
    keys = argmax_keys(vals, idx)
    order = torch.argsort(keys, descending=True)
    # 3.0 at index 2 beats 3.0 at index 6; -0.0 (index 1) and +0.0 (index 9) are equal values.
    assert idx[order].tolist() == [2, 6, 4, 1, 9, 7]
    assert torch.equal(key_index(keys), idx)
