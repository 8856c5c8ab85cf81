"""Multi-GPU arms of bench.py (imported by it; not part of the hexgen2_b200 package).

  run_serving  (bench.py --gpus N, N > 1; --workload serve | llama70b)
      Disaggregated serving through hexgen2_b200.serving: prefill groups stream every request's
      KV over NVLink into decode groups' continuous batchers.
      serve:    BASELINE config 3 (Llama-2-7B arch, bf16), weak scaling: every decode group
                serves `--batch` requests (the bench's seeded lognormal prompts) per step to
                `--out-len` tokens; `--split P:tp` fixes the split (config 3's 2:2 on 4 GPUs),
                by default about one prefill GPU per three decode GPUs (Split.for_throughput).
      llama70b: Llama-2-70B arch, prefill TP = decode TP = N / 2 (TP4 + TP4 on
                8 GPUs), `--requests` Poisson arrivals at `--rate` per second, prompts
                uniform [256, 2048], outputs uniform [64, 512].
      value = generated tokens of the timed requests / the timed region's device time (CUDA
      events on every rank between two barriers, max over ranks): the serving system's output
      token throughput, prefill included, as at N = 1.
  run_kv_bench (bench.py --workload kv_handoff)
      KV-cache handoff microbenchmark on the Llama-2-70B cache geometry.
  run_peer_copy (bench.py --workload peer_copy)
      The NVLink peer-copy figure the KV-handoff fractions are quoted against.
"""
from __future__ import annotations

import os
import statistics
import time
from datetime import timedelta

import torch
import torch.distributed as dist

NVLINK_PEER_GBS = 778.0     # measured peer copy per direction, one GPU pair (`--workload peer_copy`)
NVLINK_NOMINAL_GBS = 900.0  # NVLink 5 per direction per GPU

LLAMA2_70B = dict(vocab_size=32000, hidden_size=8192, intermediate_size=28672,
                  num_hidden_layers=80, num_attention_heads=64, num_key_value_heads=8,
                  rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=4096)


def _quiet_nccl():
    """NCCL's version banner would land on stdout next to the bench's one JSON line."""
    if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
        os.environ["NCCL_DEBUG"] = "WARN"


def _init():
    _quiet_nccl()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=600),
                            device_id=torch.device("cuda", local))
    return local


def _max(values):
    t = torch.tensor(values, dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.cpu().tolist()


def _sum(values):
    t = torch.tensor(values, dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.cpu().tolist()


def _pct(xs, q):
    xs = sorted(xs)
    return round(xs[min(len(xs) - 1, int(q * len(xs)))], 2) if xs else None


# ------------------------------------------------------------------------------------------
# Disaggregated serving
# ------------------------------------------------------------------------------------------
def _closed_loop(split, prompts, out_len, steps, rid0):
    """`steps` batches of the same prompts for every decode group; request ids interleave the
    decode groups so a prefill group feeding several of them fills them evenly."""
    from hexgen2_b200.serving import Request
    B, nd = len(prompts), split.n_decode_groups
    reqs = []
    for s in range(steps):
        for b, p in enumerate(prompts):
            for j in range(nd):
                rid = rid0 + (s * B + b) * nd + j
                reqs.append(Request(rid, p, out_len, 0.0, group=j, index=s * B + b))
    return reqs


def _poisson(n, rate, seed, vocab, rid0=0):
    from hexgen2_b200.serving import Request
    g = torch.Generator().manual_seed(seed + 7)
    gaps = torch.empty(n, dtype=torch.float64).exponential_(rate, generator=g)
    arrivals = (torch.cumsum(gaps, 0) - gaps[0]).tolist()
    plens = torch.randint(256, 2049, (n,), generator=g).tolist()
    olens = torch.randint(64, 513, (n,), generator=g).tolist()
    return [Request(rid0 + i, torch.randint(0, vocab, (plens[i],), generator=g).tolist(), olens[i],
                    arrivals[i]) for i in range(n)]


def run_serving(args, bench) -> dict | None:
    from hexgen2_b200 import ops
    from hexgen2_b200.engine import Engine
    from hexgen2_b200.serving import (DecodeWorker, PrefillWorker, Split, assign, connect_rings,
                                      make_groups)
    local = _init()
    rank, world = dist.get_rank(), dist.get_world_size()
    poisson = args.workload == "llama70b"
    if poisson:
        cfg = dict(LLAMA2_70B)
        split = Split(world, world // 2, world // 2)
    else:
        cfg = dict(bench.LLAMA2_7B)
        if args.split:
            p, tp = (int(x) for x in args.split.split(":"))
            split = Split(world, p, tp)
        else:
            split = Split.for_throughput(world)
    if args.layers:
        cfg["num_hidden_layers"] = args.layers  # small test runs only (the line says so)
    group = make_groups(split)
    kind, gidx, tpi = split.role(rank)
    eng = Engine.from_config(cfg, dtype="bfloat16", seed=args.seed, process_group=group)
    store = dist.PrefixStore(f"hx-serve-{args.seed}", dist.distributed_c10d._get_default_store())
    dev = eng.device

    if poisson:
        warm = assign(_poisson(4, 1e6, args.seed + 1, cfg["vocab_size"], rid0=10 ** 6), split)
        timed = assign(_poisson(args.requests, args.rate, args.seed, cfg["vocab_size"]), split)
        e2e_reqs = []
        slots, capacity, max_prompt = args.batch, 2048 + 512 + 1, 2048
        prompts = None
    else:
        prompts = bench.make_prompts(args.batch, args.seed, cfg["vocab_size"])
        warm = _closed_loop(split, prompts, args.out_len, args.warmup, 0)
        timed = _closed_loop(split, prompts, args.out_len, args.steps, 10 ** 6)
        e2e_reqs = _closed_loop(split, prompts, args.out_len, args.e2e_steps, 2 * 10 ** 6)
        slots = args.batch
        max_prompt = max(len(p) for p in prompts)
        capacity = max_prompt + args.out_len
    per_token = eng.num_layers * eng.row_bytes
    ring_bytes = int(args.ring_gb * 2 ** 30) if args.ring_gb else min(
        24 * 2 ** 30, max(4 * max_prompt * per_token, int(1.25 * slots * 1100 * per_token)))
    handoffs, staging, remotes = connect_rings(split, ring_bytes)
    if kind == "prefill":
        worker = PrefillWorker(eng, split, store, remotes, ring_bytes, max_prompt)
    else:
        worker = DecodeWorker(eng, split, store, staging, slots, capacity)
    device_ids = None
    if prompts is not None and kind == "prefill":
        uniq, device_ids = {}, {}
        for r in warm + timed:
            key = id(r.prompt)
            if key not in uniq:
                uniq[key] = torch.tensor([r.prompt], dtype=torch.long, device=dev)
            device_ids[r.rid] = uniq[key]

    def phase(reqs, prefix, ids):
        torch.cuda.synchronize()
        dist.barrier()
        t0 = time.monotonic()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = worker.run(reqs, prefix, t0, ids) if kind == "prefill" else worker.run(reqs, prefix, t0)
        e1.record()
        torch.cuda.synchronize()
        wall = time.monotonic() - t0
        dist.barrier()
        return out, e0.elapsed_time(e1), wall

    phase(warm, "w", device_ids)
    worker.stats.clear()
    if kind == "decode":
        worker.step_times.clear()
    ops.LAUNCHES = 0
    with bench.ClockSampler(local, enabled=args.clocks) as clocks:
        outputs, dev_ms, _ = phase(timed, "t", device_ids)
    launches = ops.LAUNCHES
    stats = list(worker.stats)
    steps_done = getattr(worker, "steps", 0)
    step_times = list(getattr(worker, "step_times", []))
    tokens_ok = _check_tokens(outputs, timed) if kind == "decode" else None

    # End to end: prompts from pinned host memory to host token lists (wall clock, max over ranks).
    e2e = None
    if e2e_reqs:
        _, _, wall = phase(e2e_reqs, "e", None)
        wall_max = _max([wall])[0]
        ntok = sum(r.max_new for r in e2e_reqs)
        e2e = {"value": round(ntok / wall_max, 2), "unit": "tokens/s",
               "what": ("generated tokens/s: prompt ids from pinned host memory on the prefill "
                        "ranks, tokens read back to host lists every decode step (wall clock "
                        "between barriers, max over ranks)"),
               "h2d_bytes_per_step": 8 * sum(len(p) for p in prompts) * split.n_decode_groups,
               "d2h_bytes_per_step": 8 * args.batch * args.out_len * split.n_decode_groups,
               "steps": args.e2e_steps}

    # Decode-step kernel classes on the first decode rank (TP1: each class alone).
    roofs = None
    if (args.profile_kernels and kind == "decode" and gidx == 0 and tpi == 0 and split.tp == 1
            and prompts):
        mid = [len(p) + args.out_len // 2 for p in prompts]
        times = bench.class_step_times(eng, worker.batcher.cache, mid, capacity)
        roofs = bench.roofline_entries(times, bench.decode_step_bytes(cfg, mid), bench.peaks())

    dev_max = _max([dev_ms])[0]
    launches_all = int(_sum([launches])[0])
    gathered = [None] * world
    dist.all_gather_object(gathered, {"kind": kind, "stats": stats, "clocks": clocks.summary(),
                                      "roofs": roofs, "steps": steps_done, "tokens_ok": tokens_ok,
                                      "step_times": _step_summary(step_times)})
    for h in handoffs:
        h.close()
    torch.cuda.synchronize()
    if kind == "decode":
        eng.release_graphs()  # they may hold NCCL collectives of this process group
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return None
    return _serving_line(args, bench, split, cfg, timed, gathered, dev_max, launches_all, e2e, poisson)


def _step_summary(times):
    """p50 / p90 of a decode rank's host time per decode step: control (store, admissions) and
    the step itself (graph replay until the tokens are read back), and the mean active slots."""
    if not times:
        return None
    ctrl = [1e3 * t[0] for t in times]
    step = [1e3 * t[1] for t in times]
    return {"steps": len(times), "control_ms_p50": _pct(ctrl, 0.5), "control_ms_p90": _pct(ctrl, 0.9),
            "step_ms_p50": _pct(step, 0.5), "step_ms_p90": _pct(step, 0.9),
            "active_slots_mean": round(sum(t[2] for t in times) / len(times), 2)}


def _check_tokens(outputs, timed):
    """Every timed request of this decode group produced max_new tokens."""
    want = {r.rid: r.max_new for r in timed}
    return all(len(v) == want[k] for k, v in outputs.items())


def _serving_line(args, bench, split, cfg, timed, gathered, dev_max, launches, e2e, poisson):
    pre = [s for g in gathered if g["kind"] == "prefill" for s in g["stats"]]
    dec = [s for g in gathered if g["kind"] == "decode" for s in g["stats"]]
    gen = sum(r.max_new for r in timed)
    value = gen / (dev_max / 1e3)
    by_rid = {r.rid: r for r in timed}
    prefill_ms = [(s["ready"] - s["start"]) * 1e3 for s in pre]
    ttft_ms = [(s["ready"] - s["arrival"]) * 1e3 for s in pre]
    kv_gbs = [s["kv_bytes"] / (s["kv_ms"] / 1e3) / 1e9 for s in pre if s["kv_ms"] > 0]
    lat_ms = [(s["done"] - by_rid[s["rid"]].arrival) * 1e3 for s in dec if s["rid"] in by_rid]
    clock_rows = [g["clocks"] for g in gathered]
    sm = [c["sm_mhz"] for c in clock_rows if c and c.get("sm_mhz")]
    reasons = sorted({x for c in clock_rows if c for x in c.get("reasons", [])})
    roofs = next((g["roofs"] for g in gathered if g["roofs"]), None)
    roofline = dict(max(roofs.values(), key=lambda r: r["ms"])) if roofs else None
    kv_med = statistics.median(kv_gbs) if kv_gbs else None
    dec_ranks = [g for g in gathered if g["kind"] == "decode"]
    steps = max((g["steps"] for g in dec_ranks), default=0)
    n_steps = 1 if poisson else args.steps
    line = {
        "metric": (bench.METRIC if not poisson else
                   "generated tokens/s + TTFT (Llama-2-70B arch, Poisson arrivals, disaggregated TP)"),
        "value": round(value, 2), "unit": "tokens/s", "n_gpus": split.world,
        "steps": n_steps, "warmup": 1 if poisson else args.warmup,
        "ms_per_step": round(dev_max / n_steps, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights, uniform token ids)",
        "value_definition": bench.VALUE_DEFINITION,
        "ttft_p50_ms": _pct(ttft_ms if poisson else prefill_ms, 0.5),
        "ttft_p90_ms": _pct(ttft_ms if poisson else prefill_ms, 0.9),
        "ttft_definition": ("first token ready on the prefill rank - request arrival (queueing "
                            "included)" if poisson else
                            "closed loop: first token ready on the prefill rank - the prefill "
                            "rank taking the request (the prefill ranks run ahead of the decode "
                            "ranks through the staging ring, so a request never waits for a "
                            "decode slot before its prefill)"),
        "ttft_queue_inclusive_ms": {"p50": _pct(ttft_ms, 0.5), "p90": _pct(ttft_ms, 0.9),
                                    "what": "first token ready - arrival (closed loop: every "
                                            "request arrives at the start of the run)"},
        "prefill_latency_ms": {"p50": _pct(prefill_ms, 0.5), "p90": _pct(prefill_ms, 0.9)},
        "request_latency_ms": {"p50": _pct(lat_ms, 0.5), "p90": _pct(lat_ms, 0.9)},
        "decode_steps_max_rank": steps,
        "decode_step_host_ms": [g["step_times"] for g in dec_ranks if g["step_times"]][:2],
        "kv_transfer_gbs_per_pair": round(kv_med, 1) if kv_med else None,
        "kv_roofline": None if not kv_med else {
            "kernel": "kv_pack (peer stores over NVLink, one request per launch)", "bound": "nvlink",
            "achieved": round(kv_med, 1), "peak": NVLINK_PEER_GBS, "unit": "GB/s",
            "frac": round(kv_med / NVLINK_PEER_GBS, 4),
            "frac_of_nominal_900": round(kv_med / NVLINK_NOMINAL_GBS, 4),
            "peak_source": "measured peer copy per direction on this pool (profiles/nvlink_peer_copy.md)"},
        "config": {"workload": (("Llama-2-70B arch (BASELINE config 4): " if poisson else
                                 "Llama-2-7B arch (BASELINE config 3), disaggregated: ") + split.describe()),
                   "model": "llama-2-70b-arch" if poisson else "llama-2-7b-arch",
                   "layers": cfg["num_hidden_layers"],
                   "split": {"prefill_gpus": split.prefill_gpus,
                             "decode_gpus": split.world - split.prefill_gpus, "tp": split.tp},
                   "requests": len(timed), "slots_per_decode_group": args.batch,
                   "parallelism": (f"prefill tp{split.tp} x {split.n_prefill_groups} + "
                                   f"decode tp{split.tp} x {split.n_decode_groups}"),
                   "l2": "inputs larger than L2 (weights + KV caches stream every step)"},
        "e2e": e2e, "gpu_launches": launches, "roofline": roofline, "rooflines": roofs,
        "clocks": {"sm_mhz": statistics.median(sm) if sm else None,
                   "sm_max_mhz": max((c.get("sm_max_mhz") or 0) for c in clock_rows if c) or None,
                   "reasons": reasons, "per_rank": clock_rows},
        "all_tokens_generated": all(g["tokens_ok"] for g in dec_ranks),
        "cpu_baseline": None,
    }
    if poisson:
        line["config"].update({"rate_per_s": args.rate, "prompt_len": "uniform [256, 2048]",
                               "output_len": "uniform [64, 512]"})
    else:
        line["config"].update({"global_batch": args.batch * split.n_decode_groups,
                               "prompt_lens_mean": round(sum(len(r.prompt) for r in timed) / len(timed), 1),
                               "output_len": args.out_len})
    return line


# ------------------------------------------------------------------------------------------
# NVLink peer-copy reference figure
# ------------------------------------------------------------------------------------------
def run_peer_copy(args) -> dict:
    """Copy-engine peer copies between GPU 0 and GPU 1 of one process (cudaMemcpyPeerAsync
    through hx_peer_copy), 1 GiB per copy: one direction alone, then both directions at once
    (two streams). GB/s = bytes per direction / CUDA-event time, best of --steps after
    --warmup. This is the per-direction NVLink figure the KV-handoff fractions divide by."""
    from hexgen2_b200 import _lib
    lib = _lib.lib()
    if torch.cuda.device_count() < 2:
        return {"workload": "peer_copy", "unavailable": "needs 2 GPUs in one process"}
    n = 1 << 30
    for d in (0, 1):
        torch.cuda.set_device(d)
        _lib.check(lib.hx_enable_peer_access(1 - d), "hx_enable_peer_access")
    a0 = torch.empty(n, dtype=torch.uint8, device="cuda:0")
    b0 = torch.empty(n, dtype=torch.uint8, device="cuda:0")
    a1 = torch.empty(n, dtype=torch.uint8, device="cuda:1")
    b1 = torch.empty(n, dtype=torch.uint8, device="cuda:1")
    s0 = torch.cuda.Stream(device=0)
    s1 = torch.cuda.Stream(device=1)

    def one(bidir):
        e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        with torch.cuda.device(0):
            e[0].record(s0)
            _lib.check(lib.hx_peer_copy(a1.data_ptr(), 1, a0.data_ptr(), 0, n, s0.cuda_stream), "peer copy")
            e[1].record(s0)
        if bidir:
            with torch.cuda.device(1):
                e[2].record(s1)
                _lib.check(lib.hx_peer_copy(b0.data_ptr(), 0, b1.data_ptr(), 1, n, s1.cuda_stream), "peer copy")
                e[3].record(s1)
        torch.cuda.synchronize(0)
        torch.cuda.synchronize(1)
        t = [e[0].elapsed_time(e[1])] + ([e[2].elapsed_time(e[3])] if bidir else [])
        return n / (max(t) / 1e3) / 1e9

    out = {}
    for bidir in (False, True):
        for _ in range(args.warmup):
            one(bidir)
        out["bidirectional" if bidir else "one_direction"] = round(max(one(bidir) for _ in range(args.steps)), 1)
    return {"workload": "peer_copy", "metric": "NVLink peer copy GB/s per direction (GPU0 <-> GPU1)",
            "value": out["one_direction"], "unit": "GB/s", "n_gpus": 2, "steps": args.steps,
            "warmup": args.warmup, "bytes_per_copy": n, "gbs_per_direction": out,
            "nominal_gbs_per_direction": NVLINK_NOMINAL_GBS}


# ------------------------------------------------------------------------------------------
# KV-cache handoff microbenchmark (Llama-2-70B cache geometry)
# ------------------------------------------------------------------------------------------
KV70B = dict(layers=80, kv_heads=8, head_dim=128, max_seq=4096)


def _positional_checksum(buf: torch.Tensor) -> tuple[int, int]:
    """(sum of 64-bit words, sum of word * (index + 1)), both mod 2^64: any changed, missing or
    misplaced 8-byte word changes the pair."""
    w = buf.view(torch.int64)
    idx = torch.arange(1, w.numel() + 1, dtype=torch.int64, device=w.device)
    return int(w.sum().item()), int((w * idx).sum().item())


def run_kv_bench(args, bench) -> dict | None:
    """Packs the live rows of a batch of requests' caches ([80 layers, max_seq 4096, 2, 8 kv
    heads, 128] bf16 each, N(0, 1), live lengths uniform in [128, 4096]) from every sender rank
    straight into its receiver's IPC-mapped buffer (one gather-pack launch per batch, peer
    stores over NVLink), all pairs at once. Pairs: rank r -> r + N/2 for r < N/2 (N/2 pairs),
    or with --kv-bidir every rank r -> (r + N/2) mod N (N pairs: each GPU sends and receives at
    once). GB/s = live bytes per pair / the slowest pair's CUDA-event time. Every request's
    bytes are checked on the receiver against the sender's local pack (positional 64-bit
    checksums). With one GPU the pack goes to local HBM (the kernel's HBM roofline)."""
    from hexgen2_b200 import ops
    from hexgen2_b200.transport import KVHandoff
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        _quiet_nccl()
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    rank = dist.get_rank() if world > 1 else 0
    if world > 1 and world % 2:
        raise ValueError("the KV handoff bench pairs ranks: use an even number of GPUs")
    P = max(1, world // 2)
    bidir = world > 1 and args.kv_bidir
    pairs = [(r, (r + P) % world) for r in range(world if bidir else P)] if world > 1 else []
    sender = world == 1 or any(s == rank for s, _ in pairs)
    g = dict(KV70B, kv_heads=args.kv_heads or KV70B["kv_heads"])
    row = 2 * g["kv_heads"] * g["head_dim"] * 2
    results = []
    for B in [int(x) for x in args.kv_batches.split(",")]:
        gen = torch.Generator().manual_seed(args.seed + B)
        lens = torch.randint(128, g["max_seq"] + 1, (B,), generator=gen).tolist()
        offs, o = [], 0
        for L in lens:
            offs.append(o)
            o += g["layers"] * L * row
        total = o
        live = torch.tensor(lens, dtype=torch.int64, device=dev)
        offs_t = torch.tensor(offs, dtype=torch.int64, device=dev)
        handoffs, dst, staging = [], None, None
        for s, d in pairs:  # one global order: deadlock-free handle exchange
            if rank == d:
                h = KVHandoff(s)
                staging = h.expose(total)
                handoffs.append(h)
            elif rank == s:
                h = KVHandoff(d)
                dst = h.attach()
                handoffs.append(h)
        if sender:
            cg = torch.Generator(device=dev).manual_seed(args.seed * 1000 + rank * 7 + B)
            cache = torch.randn(g["layers"], B, g["max_seq"], 2, g["kv_heads"], g["head_dim"],
                                generator=cg, device=dev, dtype=torch.bfloat16)
            src = torch.tensor([cache.data_ptr() + b * cache.stride(1) * 2 for b in range(B)],
                               dtype=torch.int64, device=dev)
            if world == 1:
                dst = torch.empty(total, dtype=torch.uint8, device=dev)

            def pack(target):
                ops.kv_pack(src, live, offs_t, g["layers"], cache.stride(0) * 2,
                            cache.stride(2) * 2, row, max(lens), target)
        for _ in range(args.warmup):
            if sender:
                pack(dst)
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
        ms = 0.0
        for _ in range(args.steps):
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            if sender:
                pack(dst)
            e1.record()
            torch.cuda.synchronize()
            ms += e0.elapsed_time(e1) if sender else 0.0
        if world > 1:
            dist.barrier()
        # Bit-exactness: per-request checksums of the bytes that arrived vs a local pack.
        sent, got = None, None
        if sender:
            tmp = torch.empty(g["layers"] * max(lens) * row, dtype=torch.uint8, device=dev)
            sent = []
            for b in range(B):
                ops.kv_pack(src[b:b + 1], live[b:b + 1], torch.zeros(1, dtype=torch.int64, device=dev),
                            g["layers"], cache.stride(0) * 2, cache.stride(2) * 2, row, lens[b], tmp)
                sent.append(_positional_checksum(tmp[:g["layers"] * lens[b] * row]))
            if world == 1:
                got = [_positional_checksum(dst[offs[b]:offs[b] + g["layers"] * lens[b] * row])
                       for b in range(B)]
            del tmp, cache
        if staging is not None:
            got = [_positional_checksum(staging[offs[b]:offs[b] + g["layers"] * lens[b] * row])
                   for b in range(B)]
        torch.cuda.synchronize()
        if world > 1:
            rows = [None] * world
            dist.all_gather_object(rows, {"sent": sent, "got": got})
            exact_all = all([list(x) for x in rows[d]["got"]] == [list(x) for x in rows[s]["sent"]]
                            for s, d in pairs)
            ms_max = _max([ms])[0]
            dist.barrier()
            for h in handoffs:
                h.close()
        else:
            ms_max, exact_all = ms, got == sent
        per_step_ms = ms_max / args.steps
        gbs_pair = total / (per_step_ms / 1e3) / 1e9
        peak = NVLINK_PEER_GBS if world > 1 else bench.peaks()["hbm_gbs"]
        # A local pack moves each byte twice through HBM (read + write); over NVLink the live
        # bytes cross the link once.
        achieved = gbs_pair if world > 1 else 2 * gbs_pair
        results.append({"batch": B, "pairs": len(pairs), "live_bytes_per_pair": total,
                        "mean_live_len": round(sum(lens) / B, 1), "ms": round(per_step_ms, 3),
                        "gbs_per_pair": round(gbs_pair, 1),
                        "gbs_aggregate": round(gbs_pair * max(1, len(pairs)), 1),
                        "frac": round(achieved / peak, 4),
                        "frac_of_nominal_900": round(gbs_pair / NVLINK_NOMINAL_GBS, 4) if world > 1 else None,
                        "bit_exact": bool(exact_all)})
        del staging
        torch.cuda.empty_cache()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None
    main = results[-1]
    return {"metric": "KV-transfer GB/s per prefill->decode pair (Llama-2-70B cache geometry)",
            "value": main["gbs_per_pair"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 bytes", "data": "synthetic N(0,1) caches",
            "config": {"workload": "KV handoff microbenchmark (BASELINE config 5)",
                       "cache_per_request": [g["layers"], g["max_seq"], 2, g["kv_heads"], g["head_dim"]],
                       "live_len": "uniform [128, 4096]",
                       "pairs": ("every GPU sends and receives" if bidir else "r -> r + N/2"),
                       "path": ("gather-pack kernel with peer stores into an IPC-mapped buffer"
                                if world > 1 else "gather-pack into local HBM")},
            "roofline": {"bound": "nvlink" if world > 1 else "hbm",
                         "achieved": main["gbs_per_pair"] if world > 1 else round(2 * main["gbs_per_pair"], 1),
                         "peak": NVLINK_PEER_GBS if world > 1 else bench.peaks()["hbm_gbs"],
                         "unit": "GB/s", "frac": main["frac"]},
            "batches": results}
