"""Benchmark: HexGen-2 prefill/decode hot path on B200 (driver contract: one JSON line).

Workload (the one the headline metric names): Llama-2-7B architecture
(32 layers, hidden 4096, 32 heads MHA, head_dim 128, intermediate 11008, vocab 32000),
random-init bf16 weights N(0, 0.02); a batch of B requests (default 32) with prompt lengths
drawn lognormal(mean 1024, sigma 0.5) clipped to [128, 4096] (mu = ln 1024 - sigma^2/2), token
ids uniform; greedy decode to 256 output tokens. One step = prefill every request (TTFT per
request) + decode the batch (ragged per-sequence lengths) to 256 tokens.
  N = 1: colocated on one GPU (prefill writes straight into the decode cache slots).
  N > 1: prefill group = ranks [0, N/2), decode group = ranks [N/2, N), tensor-parallel
         (TP = N/2) inside each group over NCCL; each prefill rank hands its KV shard to decode
         rank r + N/2 over NVLink (IPC-mapped buffer written by the gather-pack kernel).

value   = decode tokens/s (tokens produced by decode steps / decode-phase device time), summed
          over the whole job; ttft_p50_ms alongside.
e2e     = the same batch through the public API (Engine.serve_batch) from pinned host token
          ids to host token lists, H2D/D2H inside the timed region: generated tokens/s.
--impl reference: the reference algorithm on the host CPU (the oracle port), bounded sample.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

LLAMA2_7B = dict(vocab_size=32000, hidden_size=4096, intermediate_size=11008,
                 num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=32,
                 rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=4096 + 512)
METRIC = "decode tokens/s + p50 TTFT (Llama-2-7B arch, bf16)"


def prompt_lengths(batch: int, seed: int) -> list[int]:
    g = torch.Generator().manual_seed(seed)
    sigma = 0.5
    mu = math.log(1024) - sigma * sigma / 2
    z = torch.randn(batch, generator=g, dtype=torch.float64)
    return [int(min(4096, max(128, round(math.exp(mu + sigma * float(v)))))) for v in z]


def make_prompts(batch: int, seed: int, vocab: int) -> list[list[int]]:
    lens = prompt_lengths(batch, seed)
    g = torch.Generator().manual_seed(seed + 1)
    return [torch.randint(0, vocab, (L,), generator=g).tolist() for L in lens]


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


class ClockSampler:
    """nvidia-smi sampling during the timed region (median SM clock, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, enabled: bool = True):
        self.index, self.rows, self.proc, self.enabled = index, [], None, enabled

    def __enter__(self):
        if not self.enabled:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None,
                    "reasons": ["unsampled" if self.enabled else "sampling disabled (--no-clocks)"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4)
                          if len(r) > 5 + i and r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows)}


# ------------------------------------------------------------------------------------------
# Native arm, N = 1 (colocated)
# ------------------------------------------------------------------------------------------
def kernel_work(cfg: dict, lens: list[int], out_len: int, steps: int) -> dict:
    """Algorithmic bytes / flops per kernel class over `steps` bench steps (for the roofline).
    decode_attention: live K and V of every sequence, every layer, every decode step (+ q, out);
    gemm_decode: every weight matrix once per decode step, plus the LM head of each prefill;
    gemm_prefill: 2 * tokens * (layer weights) per prompt; prefill_attention: 4 * hq * d * L^2 / 2
    per layer (causal)."""
    h, I, V, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"], cfg["num_hidden_layers"]
    hq, hk = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    d = cfg.get("head_dim") or h // hq
    B = len(lens)
    layer_params = (hq + 2 * hk) * d * h + h * hq * d + 2 * I * h + h * I
    dec_bytes = 0
    for s in range(out_len - 1):
        for Lb in lens:
            dec_bytes += 2 * hk * d * (Lb + s + 1) * 2 + 2 * hq * d * 2
    dec_bytes *= L
    gemm_dec_bytes = (out_len - 1) * (L * layer_params + V * h) * 2 + B * V * h * 2
    gemm_pre_flops = sum(2 * Lb * L * layer_params for Lb in lens)
    attn_pre_flops = sum(4 * hq * d * Lb * Lb / 2 * L for Lb in lens)
    return {"decode_attention": {"bytes": dec_bytes * steps},
            "gemm_decode": {"bytes": gemm_dec_bytes * steps},
            "gemm_prefill": {"flops": gemm_pre_flops * steps},
            "prefill_attention": {"flops": attn_pre_flops * steps}}


def rooflines(per_kernel: dict, work: dict, pk: dict) -> dict:
    out = {}
    for name, w in work.items():
        if name not in per_kernel:
            continue
        ms, n = per_kernel[name]
        if "bytes" in w:
            achieved = w["bytes"] / (ms / 1e3) / 1e9
            peak, unit, bound = pk["hbm_gbs"], "GB/s", "hbm"
        else:
            achieved = w["flops"] / (ms / 1e3) / 1e12
            peak, unit, bound = pk["bf16_tflops"], "TFLOP/s", "tensor"
        out[name] = {"kernel": name, "bound": bound, "achieved": round(achieved, 1), "peak": peak,
                     "unit": unit, "frac": round(achieved / peak, 4), "traffic": None,
                     "peak_source": pk["source"], "launches": n, "total_ms": round(ms, 2),
                     "avg_launch_us": round(ms * 1e3 / n, 2),
                     "timing": "CUDA events around every launch (graph nodes inside the decode graph), instrumented pass of the timed steps"}
    return out


def run_native_single(args) -> dict:
    import hexgen2_b200 as hx
    from hexgen2_b200 import ops
    from hexgen2_b200.gpt import CacheState

    torch.cuda.set_device(0)
    cfg = dict(LLAMA2_7B)
    eng = hx.Engine.from_config(cfg, dtype="bfloat16", seed=args.seed)
    model = eng.model
    B, out_len = args.batch, args.out_len
    prompts = make_prompts(B, args.seed, cfg["vocab_size"])
    lens = [len(p) for p in prompts]
    capacity = max(lens) + out_len
    cache = model.allocate_inference_cache(B, capacity)
    ids_dev = [torch.tensor([p], dtype=torch.long, device="cuda") for p in prompts]
    first = torch.empty(B, dtype=torch.long, device="cuda")
    lengths = torch.empty(B, dtype=torch.int32, device="cuda")
    lens_dev = torch.tensor(lens, dtype=torch.int32, device="cuda")

    def one_step(ttft_events, use_graph=True):
        for b in range(B):
            st = CacheState(capacity, max_batch_size=B, batch_size_offset=b,
                            key_value_memory_dict=cache)
            logits = model(ids_dev[b], inference_params=st, last_token_only=True).logits
            ops.argmax(logits, out=first[b:b + 1])
            if ttft_events is not None:
                ttft_events[b].record()
        lengths.copy_(lens_dev)
        dec0 = torch.cuda.Event(enable_timing=True)
        dec1 = torch.cuda.Event(enable_timing=True)
        dec0.record()
        toks = eng.decode_batch(first, cache, lengths, out_len - 1, use_graph=use_graph)
        dec1.record()
        return toks, dec0, dec1

    for _ in range(args.warmup):
        one_step(None)
    torch.cuda.synchronize()

    ops.LAUNCHES = 0
    step_marks, ttfts, decs = [], [], []
    with ClockSampler(0, enabled=args.clocks) as clocks:
        torch.cuda.synchronize()
        if args.profile_region:
            torch.cuda.cudart().cudaProfilerStart()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            s0 = torch.cuda.Event(enable_timing=True)
            s0.record()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(B)]
            toks, d0, d1 = one_step(ev)
            step_marks.append(s0)
            ttfts.append(ev)
            decs.append((d0, d1))
        t1.record()
        torch.cuda.synchronize()
        if args.profile_region:
            torch.cuda.cudart().cudaProfilerStop()
    launches = ops.LAUNCHES
    # Per-kernel durations: the same steps again, every kernel bracketed by CUDA events on the
    # launching stream; inside the decode graph the events are graph nodes and are read after
    # each replay (so no host submission gap is ever inside a measured interval).
    prof = None
    if args.profile_kernels:
        ops.PROFILE = []
        for _ in range(args.steps):
            one_step(None)
        torch.cuda.synchronize()
        prof = ops.profile_durations(ops.PROFILE)
        ops.PROFILE = None
    total_ms = t0.elapsed_time(t1)
    dec_ms = sum(a.elapsed_time(b) for a, b in decs)
    ttft_ms = [s.elapsed_time(e) for s, evs in zip(step_marks, ttfts) for e in evs]
    dec_tokens = B * (out_len - 1) * args.steps
    value = dec_tokens / (dec_ms / 1e3)

    # Per-kernel device time over the timed region.
    per_kernel, per_shape = {}, {}
    if prof:
        for name, t in prof:
            k = per_shape.setdefault(name, [0.0, 0])
            k[0] += t
            k[1] += 1
            base = name.split("[")[0]
            k = per_kernel.setdefault(base, [0.0, 0])
            k[0] += t
            k[1] += 1
    work = kernel_work(cfg, lens, out_len, args.steps)
    pk = peaks()
    roofs = rooflines(per_kernel, work, pk)
    roofline = max(roofs.values(), key=lambda r: r["total_ms"]) if roofs else None

    # End to end through the public API: pinned host prompts in, host token lists out.
    e2e = run_e2e(eng, prompts, out_len, args) if args.e2e_steps > 0 else None

    # Serial reference-algorithm baseline on the host cores (bounded sample).
    cpu = cpu_baseline(args) if args.cpu_baseline else None
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights, uniform token ids, lognormal prompt lengths)",
        "ttft_p50_ms": round(statistics.median(ttft_ms), 2),
        "config": {"workload": "Llama-2-7B arch colocated on 1 GPU (BASELINE config 3, 1-GPU sweep)",
                   "model": "llama-2-7b-arch", "batch": B, "prompt_lens_mean": round(sum(lens) / B, 1),
                   "prompt_lens_minmax": [min(lens), max(lens)], "output_len": out_len,
                   "parallelism": "colocated prefill+decode, TP1",
                   "l2": "inputs larger than L2 (13.5 GB weights + KV caches stream every step)"},
        "e2e": e2e, "gpu_launches": launches, "roofline": roofline, "rooflines": roofs,
        "clocks": clocks.summary(), "cpu_baseline": cpu,
        "decode_ms_per_step": [round(a.elapsed_time(b), 2) for a, b in decs],
        "kernel_ms": {k: round(v[0], 2) for k, v in sorted(per_kernel.items(), key=lambda kv: -kv[1][0])},
        "gemm_decode_us": {k.split("[")[1][:-1]: round(v[0] * 1e3 / v[1], 2)
                           for k, v in per_shape.items() if k.startswith("gemm_decode[")},
    }
    return line


def run_e2e(eng, prompts, out_len, args) -> dict:
    B = len(prompts)
    flat = [t for p in prompts for t in p]
    host = torch.tensor(flat, dtype=torch.long).pin_memory()
    for _ in range(1):
        eng.serve_batch(host, [len(p) for p in prompts], out_len)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.e2e_steps):
        out = eng.serve_batch(host, [len(p) for p in prompts], out_len)
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    assert len(out) == B and all(len(o) == out_len for o in out)
    return {"value": round(B * out_len * args.e2e_steps / (ms / 1e3), 2), "unit": "tokens/s",
            "what": "generated tokens/s through Engine.serve_batch (prefill + decode, host in/out)",
            "h2d_bytes_per_step": host.numel() * 8, "d2h_bytes_per_step": B * out_len * 8,
            "steps": args.e2e_steps}


# ------------------------------------------------------------------------------------------
# Reference algorithm on the CPU (the oracle port): bounded sample, extrapolated per layer.
# ------------------------------------------------------------------------------------------
def cpu_baseline(args, threads=None) -> dict:
    from oracle.llama_ref import LlamaShape, OracleModel, random_native_state

    if threads:
        torch.set_num_threads(threads)
    cores = torch.get_num_threads()
    cfg = LLAMA2_7B
    shape = LlamaShape.from_hf(cfg)
    shape.num_layers = 1
    state = random_native_state(shape, seed=args.seed, dtype=torch.bfloat16)
    model = OracleModel(shape, state, torch.bfloat16, attention="torch")
    prompts = make_prompts(args.batch, args.seed, cfg["vocab_size"])
    prompt = prompts[0][:512]
    steps = 3
    t0 = time.perf_counter()
    first, cache, _ = model.prefill(prompt, steps + 1)
    t1 = time.perf_counter()
    model.decode(first, cache, len(prompt), steps + 1)
    t2 = time.perf_counter()
    # One layer measured; the 7B model has 32 (embedding and LM head are small next to them,
    # their share is added from one extra LM-head timing).
    lm = torch.randn(1, cfg["hidden_size"]).bfloat16()
    w = state["lm_head.weight"]
    t3 = time.perf_counter()
    for _ in range(3):
        torch.nn.functional.linear(lm, w)
    lm_s = (time.perf_counter() - t3) / 3
    layer_decode_s = (t2 - t1) / steps - lm_s
    per_token_s = cfg["num_hidden_layers"] * layer_decode_s + lm_s
    prefill_s = cfg["num_hidden_layers"] * ((t1 - t0) - lm_s) + lm_s
    return {"value": round(1.0 / per_token_s, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": (f"oracle (reference algorithm, torch CPU bf16) on 1 of 32 Llama-2-7B layers: "
                       f"prefill {len(prompt)} tokens + {steps} decode steps at batch 1, extrapolated "
                       f"to 32 layers + LM head"),
            "prefill_ms_extrapolated": round(prefill_s * 1e3, 1)}


def run_reference(args) -> dict:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    cpu = cpu_baseline(args, threads=threads)
    return {"metric": METRIC, "value": cpu["value"], "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": "Llama-2-7B arch (BASELINE config 3), CPU sample",
                       "model": "llama-2-7b-arch", "batch": 1},
            "cpu_baseline": cpu,
            "e2e": {"value": cpu["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


# ------------------------------------------------------------------------------------------
# Single-kernel mode (--kernel): one entry point alone at one shape, for roofline numbers and
# for ncu captures that must stay small (a few GB on the device).
# ------------------------------------------------------------------------------------------
def run_kernel(args) -> dict:
    from hexgen2_b200 import ops

    torch.cuda.set_device(0)
    pk = peaks()
    g = torch.Generator(device="cuda").manual_seed(args.seed)
    dt = torch.bfloat16
    l2 = 126 * 2 ** 20
    iters = args.iters

    def timed(fn, n):
        # Warm-up launches size every scratch buffer; the timed launches are captured in one
        # CUDA graph so host-side launch cost is not part of the per-kernel time.
        for i in range(5):
            fn(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(n):
                fn(i)
        graph.replay()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        graph.replay()
        t1.record()
        torch.cuda.synchronize()
        return t0.elapsed_time(t1) * 1e3 / n  # us per call

    if args.kernel == "gemm":
        M, N, K = (int(v) for v in args.shape.split(","))
        epi = {"none": ops.HX_EPI_NONE, "residual": ops.HX_EPI_RESIDUAL,
               "swiglu": ops.HX_EPI_SWIGLU}[args.epi]
        wbytes = N * K * 2
        copies = max(1, min(64, -(-3 * l2 // wbytes)))  # weights rotate through > L2
        ws = [torch.randn(N, K, generator=g, device="cuda", dtype=dt) * 0.02 for _ in range(copies)]
        x = torch.randn(M, K, generator=g, device="cuda", dtype=dt)
        n_out = N // 2 if epi == ops.HX_EPI_SWIGLU else N
        out = torch.empty(M, n_out, device="cuda", dtype=dt)
        res = torch.randn(M, n_out, generator=g, device="cuda", dtype=dt) if epi == ops.HX_EPI_RESIDUAL else None
        us = timed(lambda i: ops.gemm(x, ws[i % copies], epi, residual=res, out=out), iters)
        nbytes = wbytes + M * K * 2 + M * n_out * 2 * (2 if res is not None else 1)
        flops = 2 * M * N * K
        gbs, tfs = nbytes / us / 1e3, flops / us / 1e6
        bound = "hbm" if M <= 64 else "tensor"
        achieved, peak = (gbs, pk["hbm_gbs"]) if bound == "hbm" else (tfs, pk["bf16_tflops"])
        return {"kernel": f"gemm {args.epi}", "shape": [M, N, K], "us": round(us, 2),
                "GB/s": round(gbs, 1), "TFLOP/s": round(tfs, 1), "bound": bound,
                "frac": round(achieved / peak, 4), "peak_source": pk["source"],
                "l2": f"{copies} weight copies rotated"}
    if args.kernel == "gemm_qkv":
        # Wqkv projection with rotary + KV-cache write fused into the epilogue (decode rows,
        # one token per sequence at positions around 1000).
        M, hq, hk, d = (int(v) for v in args.shape.split(","))
        h, N = hq * d, (hq + 2 * hk) * d
        wbytes = N * h * 2
        copies = max(1, min(64, -(-3 * l2 // wbytes)))
        ws = [torch.randn(N, h, generator=g, device="cuda", dtype=dt) * 0.02 for _ in range(copies)]
        x = torch.randn(M, h, generator=g, device="cuda", dtype=dt)
        cap = 1200
        pos = torch.randint(900, 1100, (M,), generator=g, device="cuda", dtype=torch.int32)
        ang = torch.arange(cap, device="cuda", dtype=torch.float32)[:, None] * \
            (1.0 / 10000 ** (torch.arange(0, d, 2, device="cuda", dtype=torch.float32) / d))
        cos, sin = ang.cos().to(dt).contiguous(), ang.sin().to(dt).contiguous()
        cache = torch.empty(M, cap, 2, hk, d, device="cuda", dtype=dt)
        q_out = torch.empty(M, hq, d, device="cuda", dtype=dt)
        us = timed(lambda i: ops.gemm_qkv_rotary(x, ws[i % copies], 1, hq, hk, d, pos, cos, sin,
                                                 cache, q_out=q_out), iters)
        nbytes = wbytes + M * h * 2 + M * N * 2
        gbs = nbytes / us / 1e3
        return {"kernel": "gemm_qkv_rotary", "shape": [M, hq, hk, d], "us": round(us, 2),
                "GB/s": round(gbs, 1), "bound": "hbm", "frac": round(gbs / pk["hbm_gbs"], 4),
                "peak_source": pk["source"], "l2": f"{copies} weight copies rotated"}
    if args.kernel == "decode_attention":
        # L = live keys of every sequence, or with --ragged the mean of the bench's lognormal
        # prompt lengths plus L (mid-decode), one length per sequence.
        B, hq, hk, d, L = (int(v) for v in args.shape.split(","))
        lens_l = [Lp + L for Lp in prompt_lengths(B, args.seed)] if args.ragged else [L] * B
        cap = max(lens_l) + 128
        cache = torch.randn(B, cap, 2, hk, d, generator=g, device="cuda", dtype=dt)
        q = torch.randn(B, hq, d, generator=g, device="cuda", dtype=dt)
        lens = torch.tensor(lens_l, dtype=torch.int32, device="cuda")
        out = torch.empty(B, hq, d, device="cuda", dtype=dt)
        us = timed(lambda i: ops.decode_attention(q, cache, lens, hk, cap, d ** -0.5, out=out), iters)
        nbytes = sum(lens_l) * 2 * hk * d * 2 + 2 * B * hq * d * 2
        gbs = nbytes / us / 1e3
        return {"kernel": "decode_attention", "shape": [B, hq, hk, d, L], "ragged": args.ragged,
                "mean_len": round(sum(lens_l) / B, 1), "us": round(us, 2),
                "GB/s": round(gbs, 1), "bound": "hbm", "frac": round(gbs / pk["hbm_gbs"], 4),
                "peak_source": pk["source"],
                "l2": f"cache {cache.numel() * 2 / 2 ** 20:.0f} MiB vs 126 MiB L2"}
    if args.kernel == "prefill_attention":
        B, hq, hk, d, S = (int(v) for v in args.shape.split(","))
        cache = torch.randn(B, S, 2, hk, d, generator=g, device="cuda", dtype=dt)
        q = torch.randn(B, S, hq, d, generator=g, device="cuda", dtype=dt)
        pos = torch.zeros(B, dtype=torch.int32, device="cuda")
        out = torch.empty_like(q)
        us = timed(lambda i: ops.prefill_attention(q, cache, pos, hk, d ** -0.5, out=out), iters)
        flops = 4 * B * hq * d * S * S / 2
        tfs = flops / us / 1e6
        return {"kernel": "prefill_attention", "shape": [B, hq, hk, d, S], "us": round(us, 2),
                "TFLOP/s": round(tfs, 1), "bound": "tensor",
                "frac": round(tfs / pk["bf16_tflops"], 4), "peak_source": pk["source"]}
    if args.kernel == "kv_pack":
        layers, hk, d, L, B = (int(v) for v in args.shape.split(","))
        cap = L + 64
        row = 2 * hk * d * 2
        big = torch.randn(layers, B, cap, 2, hk, d, generator=g, device="cuda", dtype=dt)
        dst = torch.empty(B * layers * L * row, dtype=torch.uint8, device="cuda")
        elem = 2
        src = torch.tensor([big.data_ptr() + b * big.stride(1) * elem for b in range(B)],
                           dtype=torch.int64, device="cuda")
        live = torch.full((B,), L, dtype=torch.int64, device="cuda")
        offs = torch.tensor([b * layers * L * row for b in range(B)], dtype=torch.int64, device="cuda")
        us = timed(lambda i: ops.kv_pack(src, live, offs, layers, big.stride(0) * elem,
                                         big.stride(2) * elem, row, L, dst), iters)
        nbytes = 2 * B * layers * L * row
        gbs = nbytes / us / 1e3
        return {"kernel": "kv_pack", "shape": [layers, hk, d, L, B], "us": round(us, 2),
                "GB/s": round(gbs, 1), "bound": "hbm", "frac": round(gbs / pk["hbm_gbs"], 4),
                "peak_source": pk["source"]}
    raise ValueError(args.kernel)


# ------------------------------------------------------------------------------------------
# Continuous batching under Poisson arrivals (one GPU)
# ------------------------------------------------------------------------------------------
def run_continuous(args) -> dict:
    """Requests arrive as a Poisson process (rate --rate per second, --requests of them;
    prompt lengths uniform in [256, 2048], output lengths uniform in [64, 512], the distributions
    of BASELINE config 4) and are served by ContinuousBatcher with --batch slots: admitted into
    free slots between decode steps, one graph replay per step for all slots. Reports generated
    tokens/s over the whole run (first arrival to last completion, wall clock) and TTFT / latency
    percentiles."""
    import hexgen2_b200 as hx

    torch.cuda.set_device(0)
    cfg = dict(LLAMA2_7B)
    eng = hx.Engine.from_config(cfg, dtype="bfloat16", seed=args.seed)
    g = torch.Generator().manual_seed(args.seed + 7)
    n = args.requests
    gaps = torch.empty(n, dtype=torch.float64).exponential_(args.rate, generator=g)
    arrivals = torch.cumsum(gaps, 0).tolist()
    plens = torch.randint(256, 2049, (n,), generator=g).tolist()
    olens = torch.randint(64, 513, (n,), generator=g).tolist()
    prompts = [torch.randint(0, cfg["vocab_size"], (L,), generator=g).tolist() for L in plens]
    batcher = hx.ContinuousBatcher(eng, slots=args.batch, capacity=2048 + 512 + 16)
    # Warm-up: a few requests at once (kernels, graph, scratch buffers).
    hx.serve_arrivals(batcher, [(f"w{i}", prompts[i], 8, 0.0) for i in range(min(4, n))])
    torch.cuda.synchronize()
    reqs = [(i, prompts[i], olens[i], arrivals[i] - arrivals[0]) for i in range(n)]
    ops_launch0 = hx.ops.LAUNCHES
    with ClockSampler(0, enabled=args.clocks) as clocks:
        t0 = time.perf_counter()
        stats = hx.serve_arrivals(batcher, reqs)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    gen = sum(len(v["tokens"]) for v in stats.values())
    ttft = sorted(v["ttft_s"] * 1e3 for v in stats.values())
    lat = sorted((v["done_s"] - r[3]) * 1e3 for r, v in zip(reqs, (stats[r[0]] for r in reqs)))

    def pct(xs, q):
        return round(xs[min(len(xs) - 1, int(q * len(xs)))], 1)

    return {"metric": "continuous batching generated tokens/s (Llama-2-7B arch, Poisson arrivals)",
            "value": round(gen / wall, 1), "unit": "tokens/s", "n_gpus": 1, "steps": 1,
            "warmup": 1, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (random-init weights, uniform token ids)",
            "config": {"workload": "continuous batching, Poisson arrivals (BASELINE config 4 length "
                                   "distributions on the Llama-2-7B arch, one GPU)",
                       "requests": n, "rate_per_s": args.rate, "slots": args.batch,
                       "prompt_len": "uniform [256, 2048]", "output_len": "uniform [64, 512]"},
            "wall_s": round(wall, 2), "generated_tokens": gen,
            "ttft_ms": {"p50": pct(ttft, 0.5), "p90": pct(ttft, 0.9), "p99": pct(ttft, 0.99)},
            "latency_ms": {"p50": pct(lat, 0.5), "p90": pct(lat, 0.9)},
            "gpu_launches": hx.ops.LAUNCHES - ops_launch0, "clocks": clocks.summary()}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--kernel", choices=["gemm", "gemm_qkv", "decode_attention", "prefill_attention",
                                         "kv_pack"],
                    help="time one kernel alone (shape via --shape) instead of the model step")
    ap.add_argument("--shape", default="32,4096,4096",
                    help="gemm: M,N,K; gemm_qkv: M,hq,hkv,d; decode_attention: B,hq,hkv,d,L; "
                         "prefill_attention: "
                         "B,hq,hkv,d,S; kv_pack: layers,hkv,d,L,B")
    ap.add_argument("--epi", choices=["none", "residual", "swiglu"], default="none")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--workload", choices=["serve", "kv_handoff", "continuous"], default="serve",
                    help="kv_handoff: the KV-cache handoff microbenchmark (70B cache geometry); "
                         "continuous: continuous batching under Poisson arrivals (one GPU)")
    ap.add_argument("--requests", type=int, default=64, help="continuous: number of requests")
    ap.add_argument("--rate", type=float, default=8.0, help="continuous: arrivals per second")
    ap.add_argument("--kv-batches", default="1,8,64",
                    help="kv_handoff: requests per transfer, comma separated")
    ap.add_argument("--ragged", action="store_true",
                    help="decode_attention: per-sequence lengths = bench prompt lengths + L")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--out-len", type=int, default=256)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--e2e-steps", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--no-profile", dest="profile_kernels", action="store_false")
    ap.add_argument("--no-clocks", dest="clocks", action="store_false",
                    help="do not sample nvidia-smi clocks (for runs under a profiler)")
    ap.add_argument("--profile-region", action="store_true",
                    help="bracket the timed region with cudaProfilerStart/Stop (for ncu)")
    args = ap.parse_args()
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.kernel:
        line = run_kernel(args)
    elif args.workload == "continuous" and args.impl == "native":
        line = run_continuous(args)
    elif args.workload == "kv_handoff" and args.impl == "native":
        from hexgen2_b200.disagg import run_kv_bench
        line = run_kv_bench(args, sys.modules[__name__])
    elif args.impl == "reference":
        line = run_reference(args)
    elif args.gpus == 1:
        line = run_native_single(args)
    else:
        from hexgen2_b200.disagg import run_bench_disaggregated
        line = run_bench_disaggregated(args, sys.modules[__name__])
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
