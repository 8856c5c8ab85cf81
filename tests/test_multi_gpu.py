"""Prefill group -> decode group across GPUs (NCCL + CUDA IPC over NVLink). Needs >= 2 GPUs;
skipped on a single-GPU box.

* The KV handoff moves bytes exactly: rank 0's gather-pack kernel writes the live rows of a
  seeded random cache straight into rank 1's IPC-mapped buffer; rank 1 regenerates the same
  cache and packs it locally; the two buffers are compared byte for byte.
* Disaggregated serving equals colocated serving: prompts prefilled on rank 0, KV handed to
  rank 1 over NVLink, ragged batch decoded there == the same batch served colocated on rank 1
  (greedy tokens identical). With 4 GPUs the same runs with tensor parallelism 2 per group.
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


def _serve_worker(rank, world, port, errors):
    try:
        _init(rank, world, port)
        from hexgen2_b200.disagg import DisaggregatedPair
        g = torch.Generator().manual_seed(5)
        prompts = [torch.randint(0, SMALL["vocab_size"], (L,), generator=g).tolist()
                   for L in (17, 130, 3, 64)]
        out_len = 9
        pair = DisaggregatedPair(SMALL, prompts, out_len, seed=3)
        if pair.is_prefill:
            pair.prefill_all(False)
        else:
            toks, _, _ = pair.decode_all(False, use_graph=True)
            got = toks.cpu().tolist()
            ref = pair.eng.serve_batch(prompts, max_new_tokens=out_len)
            assert got == ref, (got, ref)
        torch.cuda.synchronize()
        dist.barrier()
        pair.close()
        dist.destroy_process_group()
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


def test_disaggregated_serving_equals_colocated_2gpu():
    _need(2)
    _run(_serve_worker, 2)


def test_disaggregated_serving_equals_colocated_tp2():
    _need(4)
    _run(_serve_worker, 4)
