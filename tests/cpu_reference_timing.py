"""CPU timing of the reference's own `hf-reference` engine beside the oracle port, on one host,
one seeded checkpoint and the same prompts (test infrastructure; not collected by pytest).

The bench's CPU arm (`bench.py --impl reference`, `cpu_baseline`) times the oracle port
(oracle/llama_ref.py) because the reference tree cannot travel to the GPU box. This script
calibrates that choice where the reference is importable: it runs the reference's engine
(hexgen2/model.py:22-121, `Engine(engine="hf-reference")`, HF eager LlamaForCausalLM at batch 1:
prefill, then greedy decode one token at a time) and the port's Engine-flow restatement
(`OracleModel.prefill` / `.decode`) on the same checkpoint and prompts, at one thread (the
reference pins one thread per rank, hexgen2/run.py:97) and at every host core.

The installed transformers (5.5) differs from the reference's pin (4.36.2) in two places the
engine touches; both shims live here, outside the reference tree:
  * LlamaConfig.rope_scaling is a dict of default RoPE parameters in 5.5, which the engine's
    guard (model.py:29) takes for RoPE scaling: the engine module sees a config whose
    rope_scaling is None when the rope type is "default".
  * past_key_values is a DynamicCache rather than a tuple of (k, v) per layer (model.py:75-76,
    :99-101, :112): prefill and decode are the engine's steps with the cache read from and
    written to DynamicCache layers.

Configs: `llama7b` (config 3 widths, bf16, batch 1; timed at 1 and `--depth`
decoder layers and extrapolated to 32, as the bench's CPU arm does), `tinyllama` (config 2,
all 22 layers, bf16, a 512-token prompt and 128 new tokens) and `fixture` (config 1, the seeded
2-layer fixture in f32, prompts of 8-32 tokens, 16 new tokens). Checkpoints have seeded random
weights and are written to a temporary directory under oracle/_ref/ (git-ignored), removed at
exit. Every figure is the median of three runs.

  python tests/cpu_reference_timing.py --reference <HexGen-2 checkout> [--config llama7b]
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from oracle.llama_ref import OracleModel, load_hf_checkpoint  # noqa: E402

WIDTHS = dict(vocab_size=32000, hidden_size=4096, intermediate_size=11008,
              num_attention_heads=32, num_key_value_heads=32, max_position_embeddings=4096,
              rms_norm_eps=1e-5, rope_theta=10000.0, bos_token_id=1, eos_token_id=2,
              tie_word_embeddings=False)
TINYLLAMA = dict(vocab_size=32000, hidden_size=2048, intermediate_size=5632,
                 num_attention_heads=32, num_key_value_heads=4, max_position_embeddings=2048,
                 rms_norm_eps=1e-5, rope_theta=10000.0, bos_token_id=1, eos_token_id=2,
                 tie_word_embeddings=False)
# name: (widths or None for the fixture, full depth, dtype, default prompts, new tokens, fit)
CONFIGS = {"llama7b": (WIDTHS, 32, "bfloat16", "285,750", 16, True),
           "tinyllama": (TINYLLAMA, 22, "bfloat16", "512", 128, False),
           "fixture": (None, 2, "float32", "8,16,32", 16, False)}


def reference_engine(ref_root: Path):
    """The reference's Engine class with the two transformers-5.5 shims."""
    sys.path.insert(0, str(ref_root))
    import hexgen2.model as hm
    from transformers import DynamicCache, LlamaConfig

    class _ConfigView:
        def __init__(self, cfg):
            self._cfg = cfg

        def __getattr__(self, name):
            return getattr(self._cfg, name)

        @property
        def rope_scaling(self):
            rs = self._cfg.rope_scaling
            return None if rs is None or rs.get("rope_type", "default") == "default" else rs

    class _ConfigLoader:
        @staticmethod
        def from_pretrained(*args, **kwargs):
            return _ConfigView(LlamaConfig.from_pretrained(*args, **kwargs))

    hm.LlamaConfig = _ConfigLoader

    class ShimmedEngine(hm.Engine):
        @torch.inference_mode()
        def prefill(self, input_ids, max_new_tokens):
            ids = torch.tensor([input_ids], dtype=torch.long, device=self.device)
            result = self.model(ids, use_cache=True)
            cache = {i: torch.stack((l.keys.transpose(1, 2), l.values.transpose(1, 2)), dim=2).contiguous()
                     for i, l in enumerate(result.past_key_values.layers)}
            logits = result.logits[:, -1]
            return logits.argmax(-1), cache, logits

        @torch.inference_mode()
        def decode(self, first_token, cache, prompt_length, max_new_tokens, on_token=None):
            token = first_token.to(self.device).reshape(1)
            generated = [int(token.item())]
            past = DynamicCache()
            for i in range(len(cache)):
                past.update(cache[i][:, :, 0].transpose(1, 2).contiguous(),
                            cache[i][:, :, 1].transpose(1, 2).contiguous(), i)
            for _ in range(max_new_tokens - 1):
                result = self.model(token[:, None], past_key_values=past, use_cache=True)
                past, logits = result.past_key_values, result.logits[:, -1]
                token = logits.argmax(-1)
                generated.append(int(token.item()))
            return generated

    return ShimmedEngine


def write_checkpoint(folder: Path, widths, layers: int, dtype, seed: int):
    if widths is None:  # the seeded correctness fixture (config 1)
        from hexgen2_b200.fixture import create
        create(folder, seed=17)
        return
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    cfg = LlamaConfig(num_hidden_layers=layers, **widths)
    model = LlamaForCausalLM(cfg).to(dtype)
    model.save_pretrained(str(folder), safe_serialization=True)
    del model


def time_engine(engine, prompts, new_tokens, reps=3):
    """Median over `reps` of the prefill ms of each prompt and of the decode ms per token after
    the first prompt, batch 1."""
    engine.prefill(prompts[0][:16], 2)  # warm-up
    pre = [[] for _ in prompts]
    dec, toks = [], None
    for _ in range(reps):
        for i, p in enumerate(prompts):
            t0 = time.perf_counter()
            tok, cache, _ = engine.prefill(p, new_tokens)
            pre[i].append((time.perf_counter() - t0) * 1e3)
            if i == 0:
                t0 = time.perf_counter()
                toks = engine.decode(tok, cache, len(p), new_tokens)
                dec.append((time.perf_counter() - t0) * 1e3 / (new_tokens - 1))
    med = lambda xs: sorted(xs)[len(xs) // 2]
    return [med(x) for x in pre], med(dec), toks


def host_info():
    info = {"os_cpu_count": os.cpu_count(), "affinity": len(os.sched_getaffinity(0)),
            "machine": platform.machine()}
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True).stdout
        for line in out.splitlines():
            k, _, v = line.partition(":")
            if k.strip() in ("Model name", "Thread(s) per core", "Core(s) per socket", "Socket(s)"):
                info[k.strip()] = v.strip()
    except OSError:
        pass
    return info


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", required=True, help="HexGen-2 checkout (hexgen2/ inside)")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="llama7b")
    ap.add_argument("--prompts", default=None, help="prompt lengths (default per config)")
    ap.add_argument("--new-tokens", type=int, default=None)
    ap.add_argument("--threads", default="1,all")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--depth", type=int, default=8, help="second depth of the per-layer fit")
    args = ap.parse_args()
    widths, full, dname, dprompts, dnew, fit = CONFIGS[args.config]
    dtype = getattr(torch, dname)
    new_tokens = args.new_tokens or dnew
    Engine = reference_engine(Path(args.reference))
    lens = [int(x) for x in (args.prompts or dprompts).split(",")]
    vocab = widths["vocab_size"] if widths else 128
    g = torch.Generator().manual_seed(args.seed + 1)
    prompts = [torch.randint(3, vocab, (L,), generator=g).tolist() for L in lens]
    threads = [os.cpu_count() if t == "all" else int(t) for t in args.threads.split(",")]
    depths = (1, args.depth) if fit else (full,)
    out = {"host": host_info(), "config": args.config, "dtype": dname, "prompts": lens,
           "new_tokens": new_tokens, "layers": full, "measured_depths": list(depths), "runs": {}}
    scratch = ROOT / "oracle" / "_ref"
    scratch.mkdir(parents=True, exist_ok=True)
    with tempfile.TemporaryDirectory(dir=scratch) as tmp:
        raw = {}
        for layers in depths:
            folder = Path(tmp) / f"L{layers}"
            write_checkpoint(folder, widths, layers, dtype, args.seed)
            for nt in threads:
                torch.set_num_threads(nt)
                ref = Engine(str(folder), engine="hf-reference", device="cpu", dtype=dname)
                r_pre, r_dec, r_tok = time_engine(ref, prompts, new_tokens)
                del ref
                shape, state = load_hf_checkpoint(folder, dtype=dtype)
                port = OracleModel(shape, state, dtype=dtype)
                p_pre, p_dec, p_tok = time_engine(port, prompts, new_tokens)
                del port, state
                raw[(layers, nt)] = {"reference": (r_pre, r_dec), "port": (p_pre, p_dec),
                                     "tokens_agree": sum(a == b for a, b in zip(r_tok, p_tok))}
                print(layers, nt, raw[(layers, nt)], flush=True)
    for nt in threads:
        row = {}
        for kind in ("reference", "port"):
            if fit:
                D = args.depth
                (pre1, dec1), (pre2, dec2) = raw[(1, nt)][kind], raw[(D, nt)][kind]
                # t(1) + (full - 1) x per-layer
                pre = [a + (full - 1) * (b - a) / (D - 1) for a, b in zip(pre1, pre2)]
                dec = dec1 + (full - 1) * (dec2 - dec1) / (D - 1)
                extra = {f"prefill_ms_measured_1_{D}_layers": [[round(x, 1) for x in pre1],
                                                               [round(x, 1) for x in pre2]],
                         f"decode_ms_measured_1_{D}_layers": [round(dec1, 2), round(dec2, 2)]}
            else:
                pre, dec = raw[(full, nt)][kind]
                extra = {}
            # One request of the first prompt's length: new_tokens / (prefill + decode).
            tps = new_tokens / ((pre[0] + (new_tokens - 1) * dec) / 1e3)
            row[kind] = {f"prefill_ms_{full}_layers": [round(x, 2) for x in pre],
                         f"decode_ms_per_token_{full}_layers": round(dec, 2),
                         "tokens_per_s_first_prompt": round(tps, 3), **extra}
        row["port_over_reference_decode"] = round(row["reference"][f"decode_ms_per_token_{full}_layers"]
                                                  / row["port"][f"decode_ms_per_token_{full}_layers"], 3)
        row["port_over_reference_prefill"] = round(sum(row["reference"][f"prefill_ms_{full}_layers"])
                                                   / sum(row["port"][f"prefill_ms_{full}_layers"]), 3)
        row["greedy_tokens_agree"] = [raw[(L, nt)]["tokens_agree"] for L in depths]
        out["runs"][str(nt)] = row
    print(json.dumps(out))


if __name__ == "__main__":
    main()
