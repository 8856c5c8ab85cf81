"""Generates the golden vectors in this folder by running the HexGen-2 reference itself.

Run from the repository root in a container where the reference checkout exists:
    python tests/golden/make_golden.py --reference <path to the HexGen-2 checkout>

What runs is the reference's own code, unchanged:
  * hexgen2.fixture.create(dir, seed=0)                       (hexgen2/fixture.py:10-17)
  * hexgen2.model.Engine.prefill / Engine.decode              (hexgen2/model.py:70-121)
    driving hexgen_core.models.gpt.GPTLMHeadModel             (models/gpt.py:420-483)
    built exactly as Engine.__init__ builds it                (hexgen2/model.py:38-68)
  * remap_state_dict_hf_llama                                  (remap_state_dict.py:14-115)
  * TorchRMSNorm                                              (modules/rms_norm.py:13-15)
  * hexgen2.transport header construction / validate_header   (hexgen2/transport.py:25-60)
Three adaptations let it run on a CPU with transformers 5.5 (none changes arithmetic):
  1. two transformers class names that hexgen_core/generation.py:17 imports are stubbed;
  2. the model is built with use_flash_attn=False, so attention runs the reference's own
     torch CrossAttention (mha.py:209-244) instead of the CUDA FlashAttention kernel;
  3. flash_attn's RotaryEmbedding keeps its cos/sin cache code (_update_cos_sin_cache) but its
     Triton kernel is replaced by the same f32 rotation evaluated with torch on the CPU.
  Engine.__init__ itself is bypassed (it requires CUDA and reads config.rope_theta, which
  transformers 5.5 moved); the object is filled with the same fields it would set.
Outputs: golden.json (+ this script). Values are exact: f32 as floats, f16/bf16 as raw 16-bit
patterns; KV caches as sha256 of their raw bytes plus shapes.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
import tempfile
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def bits(t: torch.Tensor):
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.float32:
        return [float(x) for x in t.flatten().tolist()]
    return t.view(torch.int16).flatten().tolist()


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def setup_reference(ref: Path):
    import transformers.generation as tg
    for name in ("GreedySearchDecoderOnlyOutput", "SampleDecoderOnlyOutput"):
        if not hasattr(tg, name):
            setattr(tg, name, type(name, (), {}))
    sys.path[:0] = [str(ref), str(ref / "hexgen"), str(ref / "hexgen/llama")]
    import flash_attn.layers.rotary as rot

    def cpu_forward(self, qkv, kv=None, seqlen_offset=0, max_seqlen=None, num_heads_q=None):
        # Same cache as the library; rotation evaluated in f32 like its Triton kernel.
        seqlen = qkv.shape[1]
        self._update_cos_sin_cache(seqlen + seqlen_offset, device=qkv.device, dtype=qkv.dtype)
        cos = self._cos_cached[seqlen_offset:seqlen_offset + seqlen].float()[None, :, None, :]
        sin = self._sin_cached[seqlen_offset:seqlen_offset + seqlen].float()[None, :, None, :]

        def rotate(x):
            xf = x.float()
            if self.interleaved:
                x0, x1 = xf[..., 0::2], xf[..., 1::2]
            else:
                x0, x1 = xf[..., : self.dim // 2], xf[..., self.dim // 2:]
            o0, o1 = x0 * cos - x1 * sin, x0 * sin + x1 * cos
            out = (torch.stack((o0, o1), -1).reshape(xf.shape) if self.interleaved
                   else torch.cat((o0, o1), -1))
            return out.to(x.dtype)

        if kv is None:  # packed qkv [B, S, 3, H, D]: rotate q and k in place
            qkv[:, :, 0] = rotate(qkv[:, :, 0])
            qkv[:, :, 1] = rotate(qkv[:, :, 1])
            return qkv
        qkv.copy_(rotate(qkv))
        kv[:, :, 0] = rotate(kv[:, :, 0])
        return qkv, kv

    rot.RotaryEmbedding.forward = cpu_forward


def build_engine(model_dir: Path, dtype: str):
    from transformers import LlamaConfig
    from hexgen2.model import Engine
    from hexgen_core.models.gpt import GPTLMHeadModel
    from llama_config_utils import llama_config_to_gpt2_config
    from load_model_parameters_utils.remap_state_dict import remap_state_dict_hf_llama
    from safetensors.torch import load_file

    eng = Engine.__new__(Engine)
    eng.device, eng.dtype = torch.device("cpu"), getattr(torch, dtype)
    eng.config = LlamaConfig.from_pretrained(model_dir, local_files_only=True)
    eng.identity = None
    eng.kind = "native"
    config = llama_config_to_gpt2_config(eng.config)
    config.n_head_kv = eng.config.num_key_value_heads
    config.rotary_emb_base = eng.config.rope_parameters["rope_theta"]
    config.use_flash_attn = False
    config.fused_bias_fc = False
    config.fused_mlp = False
    config.fused_dropout_add_ln = False
    config.use_torch_rms_norm = True
    config.sequence_parallel = False
    eng.model = GPTLMHeadModel(config, device=eng.device, dtype=eng.dtype).eval()
    state = {}
    for shard in sorted(Path(model_dir).glob("*.safetensors")):
        state.update(load_file(str(shard), device="cpu"))
    eng.model.load_state_dict(remap_state_dict_hf_llama(state, config), strict=True)
    return eng


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", type=Path, required=True)
    ap.add_argument("--output", type=Path, default=HERE / "golden.json")
    args = ap.parse_args()
    setup_reference(args.reference)
    torch.set_num_threads(1)
    from hexgen2.fixture import create
    from hexgen2.transport import validate_header
    from transformers import LlamaForCausalLM
    from safetensors.torch import load_file

    out = {"generator": "tests/golden/make_golden.py", "fixture_seed": 0}
    with tempfile.TemporaryDirectory() as tmp:
        model_dir = Path(tmp) / "model"
        create(model_dir, seed=0)
        raw = {}
        for shard in sorted(model_dir.glob("*.safetensors")):
            raw.update(load_file(str(shard)))
        out["fixture_config"] = json.loads((model_dir / "config.json").read_text())
        out["fixture_tensor_sha256"] = {k: sha(v) for k, v in sorted(raw.items())}

        # Prompts: validate.py:22-23 cases, the tiny trace, and seeded config-1 prompts.
        cases = [{"name": f"validate-{n}", "prompt": list(range(1, n + 1)), "max_new": m}
                 for n, m in [(1, 1), (4, 4), (7, 3)]]
        trace = (args.reference / "configs/tiny-trace.jsonl").read_text().splitlines()
        for line in trace:
            if line.strip():
                row = json.loads(line)
                cases.append({"name": "trace-" + row["id"], "prompt": row["input_ids"],
                              "max_new": row["max_new_tokens"]})
        g = torch.Generator().manual_seed(0)
        for i in range(4):
            length = int(torch.randint(8, 33, (1,), generator=g))
            prompt = torch.randint(0, 128, (length,), generator=g).tolist()
            cases.append({"name": f"config1-{i}", "prompt": prompt, "max_new": 16})
        out["engine"] = {}
        for dtype in ("float32", "bfloat16", "float16"):
            eng = build_engine(model_dir, dtype)
            hf = LlamaForCausalLM.from_pretrained(model_dir, local_files_only=True,
                                                  dtype=getattr(torch, dtype),
                                                  attn_implementation="eager").eval()
            rows = []
            for case in cases:
                first, cache, logits = eng.prefill(case["prompt"], case["max_new"])
                tokens = eng.decode(first, {k: v.clone() for k, v in cache.items()},
                                    len(case["prompt"]), case["max_new"])
                ids = torch.tensor([case["prompt"]])
                hf_tokens = []
                with torch.inference_mode():
                    hf_logits = hf(ids).logits[:, -1]
                    for _ in range(case["max_new"]):
                        tok = hf(ids).logits[:, -1].argmax(-1)
                        hf_tokens.append(int(tok))
                        ids = torch.cat((ids, tok[:, None]), dim=1)
                rows.append({**case, "first_token": int(first), "tokens": tokens,
                             "prefill_logits": bits(logits[0]),
                             "kv": {str(k): {"shape": list(v.shape), "sha256": sha(v)}
                                    for k, v in cache.items()},
                             "kv_layer0_values": bits(cache[0]) if len(case["prompt"]) <= 8 else None,
                             "hf_eager_tokens": hf_tokens,
                             "hf_eager_max_logit_diff": float((hf_logits.float() - logits.float()).abs().max())})
            out["engine"][dtype] = rows

    # TorchRMSNorm KAT (tests/test_native_norm.py:15-20 inputs: seed 7, [1, 7, 128]).
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "native_norm", args.reference / "hexgen/hexgen_core/modules/rms_norm.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    torch.manual_seed(7)
    norm_rows = []
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        native = mod.TorchRMSNorm(128, dtype=dtype)
        with torch.no_grad():
            native.weight.copy_((torch.arange(128) % 7 * 0.25 + 0.5).to(dtype))
        data = torch.randn(1, 7, 128).to(dtype)
        norm_rows.append({"dtype": str(dtype), "eps": native.eps, "weight": bits(native.weight),
                          "input": bits(data), "output": bits(native(data))})
    out["rmsnorm"] = norm_rows

    # Transport packet header KAT: the pilot packet for trace-short at fp16 / bf16 / fp32.
    packets = []
    for dtype in ("float16", "bfloat16", "float32"):
        L = 4
        tensors = {"first": torch.zeros(1, dtype=torch.long),
                   **{str(i): torch.zeros(1, L, 2, 2, 32, dtype=getattr(torch, dtype))
                      for i in range(2)}}
        header = {"version": 1, "metadata": {"id": "short", "prompt_length": L}, "tensors": [
            {"name": name, "shape": list(t.shape), "dtype": str(t.dtype)} for name, t in tensors.items()]}
        packets.append({"dtype": dtype, "header": header, "payload_bytes": validate_header(header),
                        "header_utf8": json.dumps(header, allow_nan=False)})
    out["transport"] = packets
    args.output.write_text(json.dumps(out, indent=1) + "\n")
    print(f"wrote {args.output} ({args.output.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
