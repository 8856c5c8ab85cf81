"""Prefill group -> decode group across GPUs (NCCL + CUDA IPC over NVLink). Needs >= 2 GPUs;
skipped on a single-GPU box.

* The KV handoff moves bytes exactly: rank 0's gather-pack kernel writes the live rows of a
  seeded random cache straight into rank 1's IPC-mapped buffer; rank 1 regenerates the same
  cache and packs it locally; the two buffers are compared byte for byte.
* Streaming disaggregated serving equals colocated serving: requests prefilled on the prefill
  group, their KV streamed one at a time over NVLink into the decode group's continuous
  batcher, tokens identical to the decode engine's own prefill + greedy decode. Splits 1 -> 1
  (2 GPUs), 1 -> 3 and TP2 -> TP2 (4 GPUs).
* Mismatched-TP KV re-shard with shards on two GPUs of one process equals the reference's
  head concat.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SMALL = dict(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=3,
             num_attention_heads=8, num_key_value_heads=4, rms_norm_eps=1e-5,
             max_position_embeddings=1024)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))


def _handoff_worker(rank, world, port, errors):
    try:
        _init(rank, world, port)
        from hexgen2_b200 import ops
        from hexgen2_b200.transport import KVHandoff
        layers, B, cap, hk, d = 4, 3, 300, 2, 64
        lens = [1, 177, 300]
        row = 2 * hk * d * 2
        offs = [0]
        for L in lens[:-1]:
            offs.append(offs[-1] + layers * L * row)
        total = offs[-1] + layers * lens[-1] * row
        dev = torch.device("cuda", rank)
        g = torch.Generator(device=dev).manual_seed(11)
        # Both ranks draw the same cache (same seed, same GPU type).
        cache = torch.randn(layers, B, cap, 2, hk, d, generator=g, device=dev, dtype=torch.bfloat16)
        src = torch.tensor([cache.data_ptr() + b * cache.stride(1) * 2 for b in range(B)],
                           dtype=torch.int64, device=dev)
        live = torch.tensor(lens, dtype=torch.int64, device=dev)
        offs_t = torch.tensor(offs, dtype=torch.int64, device=dev)
        h = KVHandoff(1 - rank)
        if rank == 0:
            remote = h.attach()
            dist.barrier()  # the receiver has filled its buffer with a marker
            ops.kv_pack(src, live, offs_t, layers, cache.stride(0) * 2, cache.stride(2) * 2, row,
                        max(lens), remote)
            h.notify(total, 1)
        else:
            staging = h.expose(total)
            staging.fill_(0xAB)
            torch.cuda.synchronize()
            dist.barrier()
            n, seq = h.wait()
            assert (n, seq) == (total, 1)
            local = torch.empty(total, dtype=torch.uint8, device=dev)
            ops.kv_pack(src, live, offs_t, layers, cache.stride(0) * 2, cache.stride(2) * 2, row,
                        max(lens), local)
            torch.cuda.synchronize()
            assert torch.equal(staging[:total], local), "handed-off KV bytes differ"
            # The packed rows are the live slices t[:, :L] of every layer, in order.
            for b, L in enumerate(lens):
                got = staging[offs[b]:offs[b] + layers * L * row].view(torch.bfloat16)
                want = cache[:, b, :L].reshape(-1)
                assert torch.equal(got, want)
        dist.barrier()
        h.close()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        errors.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def _serve_worker(rank, world, port, errors, split_args=(1, 1)):
    """Streams requests of varied prompt and output lengths through the disaggregated pipeline
    (hexgen2_b200.serving) twice and checks, on every decode rank, that each request's tokens
    equal the same engine's own colocated prefill + greedy decode of that request."""
    try:
        import time
        _init(rank, world, port)
        from hexgen2_b200.engine import Engine
        from hexgen2_b200.serving import (DecodeWorker, PrefillWorker, Request, Split, assign,
                                          connect_rings, make_groups)
        split = Split(world, *split_args)
        group = make_groups(split)
        kind, j, t = split.role(rank)
        eng = Engine.from_config(SMALL, dtype="bfloat16", seed=3, process_group=group)
        g = torch.Generator().manual_seed(5)
        shapes = [(17, 9), (130, 4), (3, 12), (64, 1), (40, 7), (90, 10), (8, 5), (200, 3)]
        reqs = assign([Request(i, torch.randint(0, SMALL["vocab_size"], (L,), generator=g).tolist(), n)
                       for i, (L, n) in enumerate(shapes)], split)
        store = dist.PrefixStore("test-serve", dist.distributed_c10d._get_default_store())
        ring = 3 * 210 * eng.num_layers * eng.row_bytes  # small ring: regions wrap and wait
        handoffs, staging, remotes = connect_rings(split, ring)
        if kind == "prefill":
            worker = PrefillWorker(eng, split, store, remotes, ring, max_prompt=210)
            for rnd in range(2):  # a second run reuses the rings and the kept graphs
                dist.barrier()
                worker.run(reqs, f"r{rnd}", time.monotonic())
                dist.barrier()
        else:
            worker = DecodeWorker(eng, split, store, staging, slots=3, capacity=220)
            for rnd in range(2):
                dist.barrier()
                got = worker.run(reqs, f"r{rnd}", time.monotonic())
                dist.barrier()
                mine = [r for r in reqs if r.group == j]
                assert set(got) == {r.rid for r in mine}
                for r in mine:
                    first, cache, _ = eng.prefill(r.prompt, r.max_new)
                    ref = eng.decode(first, cache, len(r.prompt), r.max_new)
                    assert got[r.rid] == ref, (rnd, r.rid, got[r.rid], ref)
        torch.cuda.synchronize()
        dist.barrier()
        for h in handoffs:
            h.close()
        if kind == "decode":
            eng.release_graphs()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        errors.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def _serve_1_3(rank, world, port, errors):
    _serve_worker(rank, world, port, errors, (1, 1))


def _serve_tp2(rank, world, port, errors):
    _serve_worker(rank, world, port, errors, (2, 2))


def _serve_tp4(rank, world, port, errors):
    _serve_worker(rank, world, port, errors, (4, 4))


def _reshard_two_devices(rank, world, port, errors):
    """Mismatched-TP re-shard with the shards on two GPUs of ONE process: packs run on the
    source's device, unpacks on the destination's (rank 0 does it all; rank 1 does nothing)."""
    try:
        if rank == 0:
            from oracle.llama_ref import concat_kv_heads
            from hexgen2_b200.transport import reshard_kv
            layers, B, cap, H, d = 2, 2, 40, 4, 64
            lens, rows = [33, 7], [1, 0]
            gen = torch.Generator().manual_seed(8)
            full = torch.randn(layers, B, cap, 2, H, d, generator=gen).bfloat16()
            src = []
            for s in range(2):  # shard s on GPU s
                shard = full[:, :, :, :, s * 2:(s + 1) * 2].contiguous().to(f"cuda:{s}")
                src.append({i: shard[i] for i in range(layers)})
            dst_big = torch.zeros(layers, B, cap, 2, H, d, dtype=torch.bfloat16, device="cuda:1")
            dst = [{i: dst_big[i] for i in range(layers)}]
            torch.cuda.set_device(0)  # the current device is not the unpack's
            reshard_kv(src, dst, rows, lens, H)
            torch.cuda.synchronize(0)
            torch.cuda.synchronize(1)
            for row, L in zip(rows, lens):
                shards = [{i: src[s][i][row:row + 1, :L].cpu() for i in range(layers)} for s in range(2)]
                whole = concat_kv_heads(shards)
                for i in range(layers):
                    assert torch.equal(dst[0][i][row:row + 1, :L].cpu(), whole[i])
    except Exception as e:
        errors.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def _run(fn, world):
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, errors)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not alive, f"ranks did not finish: {msgs}"
    assert all(p.exitcode == 0 for p in procs), msgs


def _need(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def test_kv_handoff_bytes_exact_over_nvlink():
    _need(2)
    _run(_handoff_worker, 2)


def test_streaming_serving_equals_colocated_2gpu():
    """1 prefill GPU -> 1 decode GPU, requests streamed one at a time through a wrapping ring."""
    _need(2)
    _run(_serve_worker, 2)


def test_streaming_serving_one_prefill_three_decode():
    """1 prefill GPU feeding 3 decode GPUs (the default split at N = 4)."""
    _need(4)
    _run(_serve_1_3, 4)


def test_streaming_serving_tp2_to_tp2():
    """Prefill TP2 -> decode TP2 (BASELINE config 3's split): leader-decided admissions keep
    the decode group's collectives in step; greedy tokens via one all-reduce of keys."""
    _need(4)
    _run(_serve_tp2, 4)


def test_streaming_serving_tp4_to_tp4():
    """Prefill TP4 on GPUs 0-3 -> decode TP4 on GPUs 4-7 (BASELINE config 4's split): every
    TP rank hands its KV-head shard to the decode rank of the same TP index; tokens equal the
    decode group's own colocated prefill + greedy decode."""
    _need(8)
    _run(_serve_tp4, 8)


def test_reshard_kv_across_two_devices():
    _need(2)
    _run(_reshard_two_devices, 2)
