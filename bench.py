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
VALUE_DEFINITION = ("generated tokens / device time of the timed steps, prefill included: the "
                    "serving system's output-token throughput (decode_phase_tokens_per_s excludes "
                    "prefill time)")


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
# DRAM bytes per algorithmic byte of each decode-step kernel class, from one ncu capture of this
# bench with 2 of the 32 layers (dram__bytes_read.sum + dram__bytes_write.sum over one decode
# step's launches of the class / the algorithmic bytes of those launches; the summary is kept
# with the other ncu summaries). bench.py cannot run ncu; it scales its own algorithmic bytes
# by these.
DRAM_PER_ALGORITHMIC = {"gemm_decode": 0.996, "decode_attention": 1.017, "rmsnorm": 0.418}
DRAM_SOURCE = "profiles/decode_step_dram_llama7b_b32.md (ncu dram__bytes_read/write, scaled)"


def layer_params(cfg: dict) -> int:
    h, I = cfg["hidden_size"], cfg["intermediate_size"]
    hq, hk = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    d = cfg.get("head_dim") or h // hq
    return (hq + 2 * hk) * d * h + h * hq * d + 2 * I * h + h * I


def decode_step_bytes(cfg: dict, lens: list[int]) -> dict:
    """Algorithmic HBM bytes of ONE decode step of a batch whose sequences hold `lens` keys,
    per kernel class (bf16):
      gemm_decode: every weight once (4 projections per layer + the LM head) + activations
                   (inputs, outputs, residual reads);
      decode_attention: the live K and V rows of every sequence in every layer + q and output;
      rmsnorm: two norms per layer and the final one, read + write of [B, h] + the weight."""
    h, I, V, nl = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"], cfg["num_hidden_layers"]
    hq, hk = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    d = cfg.get("head_dim") or h // hq
    B, e = len(lens), 2
    qkv = (hq + 2 * hk) * d
    acts = (B * h + B * hq * d + B * qkv) + (B * hq * d + 2 * B * h) + (B * h + B * I) + (B * I + 2 * B * h)
    gemm = nl * (layer_params(cfg) * e + acts * e) + V * h * e + B * h * e + B * V * e
    attn = nl * (sum(lens) * 2 * hk * d * e + 2 * B * hq * d * e)
    norm = (2 * nl + 1) * (2 * B * h * e + h * e)
    return {"gemm_decode": gemm, "decode_attention": attn, "rmsnorm": norm}


def class_step_times(eng, cache, lens_mid: list[int], capacity: int, reps: int = 8) -> dict:
    """Device time of one decode step's launches of each kernel class, each class alone: the
    class's launches of one decode step (every layer, the model's own weights, the bench's own
    cache at the given live lengths, batch B) are captured in one CUDA graph in step order, so
    the programmatic-dependent-launch edges between consecutive launches are kept, and the
    graph is replayed `reps` times between two CUDA events on the launching stream. No event
    sits between kernels. Returns {class: (ms per decode step, launches)}."""
    from hexgen2_b200 import ops
    m = eng.model
    dev, dt = eng.device, eng.dtype
    B = len(lens_mid)
    h, hq, hk, d = m.hidden, m.hq, m.hk, m.head_dim
    layers = m.transformer.layers
    I2 = layers[0].mlp.fc1.weight.shape[0]
    g = torch.Generator(device=dev).manual_seed(3)

    def rnd(*size):
        return (torch.randn(*size, generator=g, device=dev, dtype=torch.float32) * 0.5).to(dt)

    normed, res, ctx, act = rnd(B, h), rnd(B, h), rnd(B, hq * d), rnd(B, I2 // 2)
    tmp = torch.empty(B, h, device=dev, dtype=dt)
    q = torch.empty(B, hq, d, device=dev, dtype=dt)
    attn_out = torch.empty(B, hq, d, device=dev, dtype=dt)
    logits = torch.empty(B, m.lm_head.weight.shape[0], device=dev, dtype=dt)
    pos = torch.tensor(lens_mid, dtype=torch.int32, device=dev) - 1
    seqlens = pos + 1
    cos, sin = m.rope_tables(capacity, dev, dt)

    def gemms():
        for i, layer in enumerate(layers):
            ops.gemm_qkv_rotary(normed, layer.mixer.Wqkv.weight, 1, hq, hk, d, pos, cos, sin,
                                cache[i], q_out=q)
            ops.gemm(ctx, layer.mixer.out_proj.weight, ops.HX_EPI_RESIDUAL, residual=res, out=tmp)
            ops.gemm(normed, layer.mlp.fc1.weight, ops.HX_EPI_SWIGLU, out=act)
            ops.gemm(act, layer.mlp.fc2.weight, ops.HX_EPI_RESIDUAL, residual=res, out=tmp)
        ops.gemm(normed, m.lm_head.weight, out=logits)

    def attention():
        for i in range(len(layers)):
            ops.decode_attention(q, cache[i], seqlens, hk, capacity, m.scale, out=attn_out)

    def norms():
        for layer in layers:
            ops.rmsnorm(res, layer.norm2.weight, m.eps, out=normed)
            ops.rmsnorm(res, layer.norm1.weight, m.eps, out=normed)
        ops.rmsnorm(res, m.transformer.ln_f.weight, m.eps, out=normed)

    out = {}
    for name, fn in (("gemm_decode", gemms), ("decode_attention", attention), ("rmsnorm", norms)):
        fn()  # sizes scratch buffers outside the capture
        torch.cuda.synchronize()
        before = ops.LAUNCHES
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        launches = ops.LAUNCHES - before
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        out[name] = (e0.elapsed_time(e1) / reps, launches)
        del graph
    return out


def roofline_entries(times: dict, work: dict, pk: dict) -> dict:
    out = {}
    for name, (ms, launches) in times.items():
        achieved = work[name] / (ms / 1e3) / 1e9
        out[name] = {"kernel": name, "bound": "hbm", "achieved": round(achieved, 1),
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                     "traffic": int(work[name] * DRAM_PER_ALGORITHMIC[name]),
                     "traffic_source": DRAM_SOURCE, "algorithmic_bytes": int(work[name]),
                     "per": "one decode step of the class (%d launches)" % launches,
                     "ms": round(ms, 4), "peak_source": pk["source"] + " (burst copy, of measured)",
                     "timing": ("CUDA events around replays of a graph of one decode step's "
                                "launches of this class alone (no event between kernels)")}
    return out


def prefill_class_times(eng, cache, lens: list[int], reps: int = 3) -> dict:
    """Tensor-core classes of ONE packed prefill pass (the bench's first pass: its prompts'
    rows concatenated, at most 8192), each class alone in a CUDA graph of its launches in pass
    order, CUDA events around replays:
      gemm_prefill:      the four projections of every layer over all rows of the pass, Wqkv
                         with its rotary + KV-cache write epilogue
                         (flops = 2 x rows x layer weights x layers);
      prefill_attention: causal attention of every prompt of the pass in every layer, over the
                         bench's own cache (flops = 4 x hq x d x L^2 / 2 per prompt and layer).
    Returns {class: (ms, launches, flops)}."""
    from hexgen2_b200 import ops
    from hexgen2_b200.engine import PREFILL_PROMPTS, PREFILL_TOKENS
    m = eng.model
    dev, dt = eng.device, eng.dtype
    n, T = 0, 0
    while n < len(lens) and n < PREFILL_PROMPTS and (n == 0 or T + lens[n] <= PREFILL_TOKENS):
        T += lens[n]
        n += 1
    plens = lens[:n]
    h, hq, hk, d = m.hidden, m.hq, m.hk, m.head_dim
    layers = m.transformer.layers
    I2 = layers[0].mlp.fc1.weight.shape[0]
    g = torch.Generator(device=dev).manual_seed(5)

    def rnd(*size):
        return (torch.randn(*size, generator=g, device=dev, dtype=torch.float32) * 0.5).to(dt)

    normed, res, ctx, act = rnd(T, h), rnd(T, h), rnd(T, hq * d), rnd(T, I2 // 2)
    tmp = torch.empty(T, h, device=dev, dtype=dt)
    q = rnd(T, hq, d)
    out = torch.empty(T, hq, d, device=dev, dtype=dt)
    meta = ops.varlen_meta(plens, list(range(n)), dev)  # built before the graph capture
    cos, sin = m.rope_tables(cache[0].shape[1], dev, dt)

    def gemms():
        for i, layer in enumerate(layers):
            # Wqkv with rotary + the KV-cache write in its epilogue, as the pass runs it.
            ops.gemm_qkv_rotary_varlen(normed, layer.mixer.Wqkv.weight, plens, list(range(n)),
                                       hq, hk, d, cos, sin, cache[i], q, meta=meta)
            ops.gemm(ctx, layer.mixer.out_proj.weight, ops.HX_EPI_RESIDUAL, residual=res, out=tmp)
            ops.gemm(normed, layer.mlp.fc1.weight, ops.HX_EPI_SWIGLU, out=act)
            ops.gemm(act, layer.mlp.fc2.weight, ops.HX_EPI_RESIDUAL, residual=res, out=tmp)

    def attention():
        for i in range(len(layers)):
            ops.prefill_attention_varlen(q, cache[i], plens, list(range(n)), hk, m.scale, out,
                                         meta=meta)

    flops = {"gemm_prefill": 2 * T * len(layers) * sum(w.numel() for w in (
                 layers[0].mixer.Wqkv.weight, layers[0].mixer.out_proj.weight,
                 layers[0].mlp.fc1.weight, layers[0].mlp.fc2.weight)),
             "prefill_attention": len(layers) * sum(4 * hq * d * L * L / 2 for L in plens)}
    res_t = {}
    for name, fn in (("gemm_prefill", gemms), ("prefill_attention", attention)):
        fn()
        torch.cuda.synchronize()
        before = ops.LAUNCHES
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        launches = ops.LAUNCHES - before
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        res_t[name] = (e0.elapsed_time(e1) / reps, launches, flops[name])
        del graph
    return res_t, n, T


def prefill_roofline_entries(times: dict, prompts: int, rows: int, pk: dict) -> dict:
    out = {}
    for name, (ms, launches, flops) in times.items():
        achieved = flops / (ms / 1e3) / 1e12
        # The pass is timed right after the seconds-long timed steps, at the power-capped
        # clock those run at, so the denominator is the sustained cuBLAS figure; the burst
        # fraction is kept beside it.
        peak = pk["bf16_tflops_sustained"]
        out[name] = {"kernel": name, "bound": "tensor", "achieved": round(achieved, 1),
                     "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "frac_of_burst": round(achieved / pk["bf16_tflops"], 4), "traffic": None,
                     "algorithmic_flops": int(flops),
                     "per": f"one packed prefill pass: {prompts} prompts, {rows} rows ({launches} launches)",
                     "ms": round(ms, 4),
                     "peak_source": pk["source"] + " (sustained cuBLAS bf16 under the power cap)",
                     "timing": ("CUDA events around replays of a graph of the pass's launches of "
                                "this class alone (no event between kernels)")}
    return out


def prefill_latency(eng, lengths=(512, 1024), reps=5) -> dict:
    """Isolated per-request prefill latency (batch 1, prompt ids already on the device, to the
    greedy first token on the device), median of `reps` CUDA-event timings after a warm-up."""
    from hexgen2_b200 import ops
    from hexgen2_b200.gpt import CacheState
    out = {}
    g = torch.Generator().manual_seed(7)
    for L in lengths:
        ids = torch.randint(0, eng.config.vocab_size, (1, L), generator=g).to(eng.device)
        cache = eng.model.allocate_inference_cache(1, L + 1)
        times = []
        for r in range(reps + 1):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            st = CacheState(L + 1, key_value_memory_dict=cache)
            tok = ops.argmax(eng.model(ids, inference_params=st, last_token_only=True).logits)
            e1.record()
            torch.cuda.synchronize()
            if r:
                times.append(e0.elapsed_time(e1))
        del tok
        out[str(L)] = round(statistics.median(times), 3)
    return out


def run_native_single(args) -> dict:
    import hexgen2_b200 as hx
    from hexgen2_b200 import ops
    from hexgen2_b200.gpt import CacheState

    torch.cuda.set_device(0)
    cfg = dict(LLAMA2_7B)
    if args.layers:
        cfg["num_hidden_layers"] = args.layers  # profiling runs only (the line says so)
    eng = hx.Engine.from_config(cfg, dtype="bfloat16", seed=args.seed)
    model = eng.model
    B, out_len = args.batch, args.out_len
    prompts = make_prompts(B, args.seed, cfg["vocab_size"])
    lens = [len(p) for p in prompts]
    capacity = max(lens) + out_len
    cache = model.allocate_inference_cache(B, capacity)
    flat_dev = torch.tensor([t for p in prompts for t in p], dtype=torch.long, device="cuda")
    first = torch.empty(B, dtype=torch.long, device="cuda")
    lengths = torch.empty(B, dtype=torch.int32, device="cuda")
    lens_dev = torch.tensor(lens, dtype=torch.int32, device="cuda")

    def one_step(ttft_events):
        # Prompts prefilled in packed passes of up to 8192 tokens (Engine.prefill_chunks).
        eng.prefill_chunks(flat_dev, lens, cache, first, events=ttft_events)
        lengths.copy_(lens_dev)
        dec0 = torch.cuda.Event(enable_timing=True)
        dec1 = torch.cuda.Event(enable_timing=True)
        dec0.record()
        toks = eng.decode_batch(first, cache, lengths, out_len - 1)
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
    total_ms = t0.elapsed_time(t1)
    dec_ms = sum(a.elapsed_time(b) for a, b in decs)
    ttft_ms = [s.elapsed_time(e) for s, evs in zip(step_marks, ttfts) for e in evs]
    gen_tokens = B * out_len * args.steps
    value = gen_tokens / (total_ms / 1e3)
    decode_phase = B * (out_len - 1) * args.steps / (dec_ms / 1e3)
    dec_step_ms = dec_ms / (args.steps * (out_len - 1))

    # End to end through the public API (pinned host prompts in, host token lists out), run
    # right after the timed steps so it sees the same allocator state.
    e2e = run_e2e(eng, prompts, out_len, args) if args.e2e_steps > 0 else None

    # Per-class device time of one decode step (each class alone, no events between kernels)
    # at the batch's mean live lengths (mid-decode), against the same step's algorithmic bytes.
    pk = peaks()
    roofs, roofline = {}, None
    if args.profile_kernels:
        mid = [L + out_len // 2 for L in lens]
        times = class_step_times(eng, cache, mid, capacity)
        roofs = roofline_entries(times, decode_step_bytes(cfg, mid), pk)
        roofline = dict(max(roofs.values(), key=lambda r: r["ms"]))
        roofline["decode_step_ms_in_situ"] = round(dec_step_ms, 4)
        roofline["classes_sum_ms"] = round(sum(r["ms"] for r in roofs.values()), 4)
        ptimes, pn, prow = prefill_class_times(eng, cache, lens)
        roofs.update(prefill_roofline_entries(ptimes, pn, prow, pk))

    latency = prefill_latency(eng) if args.profile_kernels else None

    # Reference algorithm on the host cores (bounded sample of the same workload).
    cpu = cpu_baseline(args, prompts, out_len) if args.cpu_baseline else None
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights, uniform token ids, lognormal prompt lengths)",
        "value_definition": VALUE_DEFINITION,
        "decode_phase_tokens_per_s": round(decode_phase, 2),
        "decode_step_ms": round(dec_step_ms, 4),
        "ttft_p50_ms": round(statistics.median(ttft_ms), 2),
        "ttft_definition": ("first token ready on the device - start of the step (the 32 prompts "
                            "are prefilled in packed passes of up to 8192 tokens, in order)"),
        "prefill_latency_ms": latency,
        "config": {"workload": "Llama-2-7B arch colocated on 1 GPU (BASELINE config 3, 1-GPU sweep)",
                   "model": "llama-2-7b-arch", "layers": cfg["num_hidden_layers"], "batch": B,
                   "prompt_lens_mean": round(sum(lens) / B, 1),
                   "prompt_lens_minmax": [min(lens), max(lens)], "output_len": out_len,
                   "parallelism": "colocated prefill+decode, TP1",
                   "l2": "inputs larger than L2 (13.5 GB weights + KV caches stream every step)"},
        "e2e": e2e, "gpu_launches": launches, "roofline": roofline, "rooflines": roofs,
        "clocks": clocks.summary(), "cpu_baseline": cpu,
        "decode_ms_per_step": [round(a.elapsed_time(b), 2) for a, b in decs],
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
# Reference algorithm on the CPU (the oracle port): the bench's own batch, one layer timed.
# ------------------------------------------------------------------------------------------
class CpuSample:
    """The reference algorithm (oracle, torch bf16 on the host cores) on ONE of the 32
    Llama-2-7B layers plus the embedding and LM head, on the bench's own workload: the same 32
    prompts prefilled one after another at batch 1 (the reference Engine's prefill), then the
    ragged batch of 32 decoded together (oracle.llama_ref.RaggedBatch). The full-model figure
    is extrapolated: 32 x the per-layer time + the embedding/LM-head time, measured apart."""

    def __init__(self, prompts, out_len, seed, threads=None):
        from oracle.llama_ref import CacheState as OCache, LlamaShape, OracleModel, RaggedBatch, random_native_state
        if threads:
            torch.set_num_threads(threads)
        self.cores = torch.get_num_threads()
        cfg = LLAMA2_7B
        self.layers = cfg["num_hidden_layers"]
        shape = LlamaShape.from_hf(cfg)
        shape.num_layers = 1
        state = random_native_state(shape, seed=seed, dtype=torch.bfloat16)
        self.model = OracleModel(shape, state, torch.bfloat16, attention="torch")
        self.lm = state["lm_head.weight"]
        self.B, self.out_len = len(prompts), out_len
        caches, lens, firsts = [], [], []
        # Untimed warm-up prefill: the first call pays one-time library set-up that the
        # 32-layer extrapolation would otherwise multiply.
        self.model.forward(torch.tensor([prompts[0]]), OCache(len(prompts[0]) + 1), last_token_only=True)
        t0 = time.perf_counter()
        for p in prompts:
            st = OCache(len(p) + out_len)
            logits = self.model.forward(torch.tensor([p]), st, last_token_only=True)
            firsts.append(int(logits.argmax(-1)))
            caches.append(st.key_value_memory_dict)
            lens.append(len(p))
        self.prefill_1layer_s = time.perf_counter() - t0
        self.batch = RaggedBatch(self.model, caches, lens)
        self.tokens = torch.tensor(firsts, dtype=torch.long)
        # LM head share of a step (it does not scale with the layer count).
        x = torch.randn(self.B, cfg["hidden_size"]).bfloat16()
        torch.nn.functional.linear(x, self.lm)  # warm-up
        t0 = time.perf_counter()
        for _ in range(3):
            torch.nn.functional.linear(x, self.lm)
        self.head_s = (time.perf_counter() - t0) / 3
        x1 = torch.randn(1, cfg["hidden_size"]).bfloat16()
        torch.nn.functional.linear(x1, self.lm)  # warm-up
        t0 = time.perf_counter()
        for _ in range(3):
            torch.nn.functional.linear(x1, self.lm)
        self.head1_s = (time.perf_counter() - t0) / 3
        self.step_s = []

    def step(self):
        t0 = time.perf_counter()
        logits = self.batch.step(self.tokens)
        self.tokens = logits.argmax(-1)
        self.step_s.append(time.perf_counter() - t0)

    def result(self, kind="port") -> dict:
        dec1 = statistics.median(self.step_s)
        dec_full = self.layers * (dec1 - self.head_s) + self.head_s
        pre_full = self.layers * (self.prefill_1layer_s - self.B * self.head1_s) + self.B * self.head1_s
        job_s = pre_full + (self.out_len - 1) * dec_full
        return {"value": round(self.B * self.out_len / job_s, 3), "unit": "tokens/s",
                "cores": self.cores, "kind": kind,
                "decode_phase_tokens_per_s": round(self.B / dec_full, 3),
                "prefill_s_extrapolated": round(pre_full, 2),
                "decode_step_s_extrapolated": round(dec_full, 4),
                "sample_step_ms": round(dec1 * 1e3, 2),
                "sample": (f"oracle (reference algorithm, torch CPU bf16, {self.cores} threads) on 1 of "
                           f"{self.layers} Llama-2-7B layers + embedding/LM head: the bench's {self.B} "
                           f"prompts prefilled one by one (batch 1), then {len(self.step_s)} decode steps "
                           f"of the ragged batch of {self.B}; extrapolated to {self.layers} layers and "
                           f"{self.out_len} output tokens (generated tokens / (prefill + "
                           f"{self.out_len - 1} decode steps))")}


def host_info() -> dict:
    info = {"os_cpu_count": os.cpu_count(), "affinity": len(os.sched_getaffinity(0)),
            "torch_threads": torch.get_num_threads()}
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for line in out.splitlines():
            if line.startswith(("Model name", "Socket(s)", "Core(s) per socket", "Thread(s) per core")):
                k, v = line.split(":", 1)
                info[k.strip()] = v.strip()
    except (OSError, subprocess.SubprocessError):
        pass
    return info


def cpu_baseline(args, prompts, out_len, threads=None) -> dict:
    sample = CpuSample(prompts, out_len, args.seed, threads=threads)
    for _ in range(2):
        sample.step()
    res = sample.result()
    res["host"] = host_info()
    return res


def run_reference(args) -> dict:
    """--impl reference: the reference algorithm on the host cores, same metric and workload
    (BASELINE config 3 at batch 32), every host thread. Each timed step is one ragged decode
    step of the one-layer sample; the line's value extrapolates to the full model and the full
    job (prefill + 255 decode steps), like cpu_baseline."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    threads = len(os.sched_getaffinity(0)) or os.cpu_count() or 1
    prompts = make_prompts(args.batch, args.seed, LLAMA2_7B["vocab_size"])
    sample = CpuSample(prompts, args.out_len, args.seed, threads=threads)
    for _ in range(args.warmup):
        sample.step()
    sample.step_s.clear()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        sample.step()
    wall = time.perf_counter() - t0
    cpu = sample.result()
    cpu["host"] = host_info()
    lens = [len(p) for p in prompts]
    return {"metric": METRIC, "value": cpu["value"], "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(wall * 1e3 / max(1, args.steps), 2),
            "ms_per_step_is": "one timed sample step (one layer of the ragged batch-32 decode step)",
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, uniform token ids, lognormal prompt lengths)",
            "impl": "reference", "value_definition": VALUE_DEFINITION,
            "config": {"workload": "Llama-2-7B arch (BASELINE config 3), host CPU, one layer timed and extrapolated",
                       "model": "llama-2-7b-arch", "batch": args.batch,
                       "prompt_lens_mean": round(sum(lens) / len(lens), 1), "output_len": args.out_len,
                       "parallelism": "host CPU threads"},
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
    ap.add_argument("--workload", choices=["serve", "llama70b", "kv_handoff", "continuous", "peer_copy"],
                    default="serve",
                    help="serve: BASELINE config 3 (Llama-2-7B), colocated at N=1, disaggregated at "
                         "N>1; llama70b: config 4 (Llama-2-70B, prefill TP=N/2 -> decode TP=N/2, "
                         "Poisson arrivals); kv_handoff: config 5 KV-cache handoff microbenchmark; "
                         "continuous: continuous batching under Poisson arrivals on one GPU; "
                         "peer_copy: NVLink peer-copy GB/s between GPU 0 and 1")
    ap.add_argument("--split", default="",
                    help="N>1 serve: 'P:tp' = P prefill GPUs, tensor-parallel groups of tp "
                         "(default: about one prefill GPU per three decode GPUs, TP1)")
    ap.add_argument("--ring-gb", type=float, default=0.0,
                    help="N>1: staging ring per decode rank in GiB (default: sized from the workload)")
    ap.add_argument("--kv-heads", type=int, default=0,
                    help="kv_handoff: KV heads per cache (default 8, the full 70B cache; 2 = one "
                         "TP4 shard)")
    ap.add_argument("--kv-bidir", action="store_true",
                    help="kv_handoff: every GPU sends to (r + N/2) mod N and receives at once")
    ap.add_argument("--requests", type=int, default=64,
                    help="continuous / llama70b: number of requests")
    ap.add_argument("--rate", type=float, default=8.0,
                    help="continuous / llama70b: Poisson arrivals per second")
    ap.add_argument("--kv-batches", default="1,8,64",
                    help="kv_handoff: requests per transfer, comma separated")
    ap.add_argument("--ragged", action="store_true",
                    help="decode_attention: per-sequence lengths = bench prompt lengths + L")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--layers", type=int, default=0,
                    help="override the layer count (small ncu captures / tests only; 0 = the model's own)")
    ap.add_argument("--out-len", type=int, default=256)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--e2e-steps", type=int, default=3)
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
    elif args.workload == "peer_copy":
        import bench_disagg
        line = bench_disagg.run_peer_copy(args)
    elif args.workload == "continuous" and args.impl == "native":
        line = run_continuous(args)
    elif args.workload == "kv_handoff" and args.impl == "native":
        import bench_disagg
        line = bench_disagg.run_kv_bench(args, sys.modules[__name__])
    elif args.impl == "reference":
        line = run_reference(args)
    elif args.gpus == 1 and args.workload == "serve":
        line = run_native_single(args)
    else:
        import bench_disagg
        line = bench_disagg.run_serving(args, sys.modules[__name__])
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
