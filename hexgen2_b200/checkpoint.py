"""Checkpoint plumbing: config mapping, HF -> native weight remap, TP sharding, random init.

Mirrors the reference's helpers (paths inside the HexGen-2 project):
  llama_config_to_gpt2_config ... hexgen/llama/llama_config_utils.py:39-67 (+ the overrides in
                                  hexgen2/model.py:48-56)
  remap_state_dict_hf_llama ..... hexgen/llama/load_model_parameters_utils/remap_state_dict.py:14-115
  shard_state_dict_tp ........... hexgen/hexgen_core/models/gpt.py:512-585
Names and layouts are the reference's, so a state dict produced by the reference's remap loads
into hexgen2_b200.gpt.GPTLMHeadModel with strict=True and vice versa.
"""
from __future__ import annotations

import hashlib
import math
import zlib
from collections import OrderedDict
from pathlib import Path

import torch


def llama_config_to_gpt2_config(llama_config):
    """HF LlamaConfig -> GPT2Config with the native model's fields (llama_config_utils.py:39-67)
    plus the attribute overrides Engine applies (hexgen2/model.py:48-56)."""
    from transformers import GPT2Config

    theta = getattr(llama_config, "rope_theta", None)
    if theta is None:
        theta = (getattr(llama_config, "rope_parameters", None) or {}).get("rope_theta", 10000.0)
    config = GPT2Config(
        vocab_size=llama_config.vocab_size, n_positions=0, n_embd=llama_config.hidden_size,
        n_layer=llama_config.num_hidden_layers, n_head=llama_config.num_attention_heads,
        n_inner=llama_config.intermediate_size, activation_function="swiglu",
        resid_pdrop=0.0, embd_pdrop=0.0, attn_pdrop=0.0,
        layer_norm_epsilon=llama_config.rms_norm_eps,
        initializer_range=llama_config.initializer_range,
        bos_token_id=llama_config.bos_token_id, eos_token_id=llama_config.eos_token_id,
        pad_token_id=llama_config.pad_token_id, rms_norm=True, rotary_emb_fraction=1.0,
        rotary_emb_interleaved=True, tie_word_embeddings=False, qkv_proj_bias=False,
        out_proj_bias=False, mlp_fc1_bias=False, mlp_fc2_bias=False)
    config.n_head_kv = llama_config.num_key_value_heads
    config.rotary_emb_base = float(theta)
    config.use_flash_attn = True
    config.fused_bias_fc = False
    config.fused_mlp = False
    config.fused_dropout_add_ln = False
    config.use_torch_rms_norm = True
    config.sequence_parallel = False
    return config


def config_from_dict(d: dict):
    """GPT2Config for a Llama architecture given as plain numbers (no checkpoint on disk)."""
    from transformers import LlamaConfig

    return llama_config_to_gpt2_config(LlamaConfig(**d))


def _pad_rows(w: torch.Tensor, multiple: int) -> torch.Tensor:
    rows = math.ceil(w.shape[0] / multiple) * multiple
    if rows == w.shape[0]:
        return w
    return torch.cat([w, w.new_zeros(rows - w.shape[0], *w.shape[1:])], dim=0)


def remap_state_dict_hf_llama(state_dict: dict, config) -> dict:
    """HF Llama names/layout -> native names/layout (remap_state_dict.py:14-115):
    fc1 = cat[up, gate]; Wqkv = cat[inv_permute(Wq), inv_permute(Wk), Wv] where inv_permute
    reorders each head's rows from (two, d/2) to (d/2, two) so rotary pairs are adjacent.
    The embedding and the LM head are zero-padded to a multiple of
    config.pad_vocab_size_multiple rows (:28-51); with config.tie_word_embeddings the LM head is
    the embedding, otherwise lm_head.weight must be present (a missing one raises KeyError,
    as in the reference)."""
    n_embd = getattr(config, "n_embd", None) or config.hidden_size
    n_head = getattr(config, "n_head", None) or config.num_attention_heads
    half = n_embd // n_head // 2
    multiple = getattr(config, "pad_vocab_size_multiple", 1) or 1
    sd = OrderedDict(state_dict)
    out = OrderedDict()
    emb = _pad_rows(sd.pop("model.embed_tokens.weight"), multiple)
    out["transformer.embeddings.word_embeddings.weight"] = emb
    if getattr(config, "tie_word_embeddings", False):
        out["lm_head.weight"] = emb
    else:
        out["lm_head.weight"] = _pad_rows(sd.pop("lm_head.weight"), multiple)
    out["transformer.ln_f.weight"] = sd.pop("model.norm.weight")

    def inv_permute(w):
        h = w.shape[0] // (2 * half)
        return w.reshape(h, 2, half, w.shape[1]).transpose(1, 2).reshape(w.shape)

    n_layer = getattr(config, "n_layer", None) or config.num_hidden_layers
    for i in range(n_layer):
        p, q = f"model.layers.{i}.", f"transformer.layers.{i}."
        out[q + "norm1.weight"] = sd.pop(p + "input_layernorm.weight")
        out[q + "norm2.weight"] = sd.pop(p + "post_attention_layernorm.weight")
        out[q + "mixer.Wqkv.weight"] = torch.cat([inv_permute(sd.pop(p + "self_attn.q_proj.weight")),
                                                 inv_permute(sd.pop(p + "self_attn.k_proj.weight")),
                                                 sd.pop(p + "self_attn.v_proj.weight")], dim=0)
        out[q + "mixer.out_proj.weight"] = sd.pop(p + "self_attn.o_proj.weight")
        out[q + "mlp.fc1.weight"] = torch.cat([sd.pop(p + "mlp.up_proj.weight"),
                                              sd.pop(p + "mlp.gate_proj.weight")], dim=0)
        out[q + "mlp.fc2.weight"] = sd.pop(p + "mlp.down_proj.weight")
        sd.pop(p + "self_attn.rotary_emb.inv_freq", None)
    for k, v in sd.items():  # anything unexpected is passed through so strict loading flags it
        out[k] = v
    return out


def shard_state_dict_tp(state_dict: dict, config, world_size: int, rank: int) -> dict:
    """Per-rank tensor-parallel slices (gpt.py:512-585): embeddings/lm_head by vocab rows,
    Wqkv by head groups, out_proj/fc2 by input columns, fc1 by the (two o) halves."""
    n_head = config.n_head
    n_head_kv = getattr(config, "n_head_kv", None) or n_head
    head_dim = config.n_embd // n_head
    assert config.vocab_size % world_size == 0 and n_head % world_size == 0
    assert n_head_kv % world_size == 0
    sd = dict(state_dict)

    def first(key):
        if key in sd:
            x = sd[key]
            d = x.shape[0] // world_size
            sd[key] = x[rank * d:(rank + 1) * d]

    def last(key):
        if key in sd:
            x = sd[key]
            d = x.shape[-1] // world_size
            sd[key] = x[..., rank * d:(rank + 1) * d]

    first("transformer.embeddings.word_embeddings.weight")
    first("lm_head.weight")
    hq, hk = n_head // world_size, n_head_kv // world_size
    for i in range(config.n_layer):
        key = f"transformer.layers.{i}.mixer.Wqkv.weight"
        if key in sd:
            x = sd[key].reshape(n_head + 2 * n_head_kv, head_dim, -1)
            sd[key] = torch.cat([x[rank * hq:(rank + 1) * hq],
                                 x[n_head + rank * hk:n_head + (rank + 1) * hk],
                                 x[n_head + n_head_kv + rank * hk:n_head + n_head_kv + (rank + 1) * hk]],
                                dim=0).reshape(-1, x.shape[-1])
        last(f"transformer.layers.{i}.mixer.out_proj.weight")
        key = f"transformer.layers.{i}.mlp.fc1.weight"
        if key in sd:
            x = sd[key]
            d = x.shape[0] // world_size // 2
            two = x.reshape(2, x.shape[0] // 2, -1)
            sd[key] = two[:, rank * d:(rank + 1) * d].reshape(-1, x.shape[-1])
        last(f"transformer.layers.{i}.mlp.fc2.weight")
    return sd


def load_safetensors_dir(model_dir) -> dict:
    """All *.safetensors shards of a checkpoint; duplicate keys are an error (model.py:58-66)."""
    from safetensors.torch import load_file

    shards = sorted(Path(model_dir).glob("*.safetensors"))
    if not shards:
        raise ValueError("A local safetensors checkpoint is required")
    state = {}
    for shard in shards:
        values = load_file(str(shard), device="cpu")
        if set(state).intersection(values):
            raise ValueError("Duplicate checkpoint keys")
        state.update(values)
    return state


def model_identity(model_dir) -> dict:
    """sha256 of config.json and of every weight shard (replaces hexgen2/record.py:42-46)."""
    model_dir = Path(model_dir)
    ident = {}
    for p in sorted(list(model_dir.glob("*.json")) + list(model_dir.glob("*.safetensors"))):
        h = hashlib.sha256()
        with p.open("rb") as f:
            for chunk in iter(lambda: f.read(1 << 20), b""):
                h.update(chunk)
        ident[p.name] = h.hexdigest()
    return ident


def _seed_for(name: str, seed: int) -> int:
    return (seed * 1000003 + zlib.crc32(name.encode())) & 0x7FFFFFFF


def random_native_state(config, seed: int = 0, dtype=torch.bfloat16, device="cuda", std=0.02,
                        tp_world: int = 1, tp_rank: int = 0) -> dict:
    """Seeded N(0, std) weights in native names, generated on `device` one tensor at a time
    (norm weights are ones). With tp_world > 1 each full tensor is generated, sliced to this
    rank's shard and freed, so every TP layout sees the same underlying model."""
    n_head = config.n_head
    n_head_kv = getattr(config, "n_head_kv", None) or n_head
    d = config.n_embd // n_head
    h, V, I = config.n_embd, config.vocab_size, config.n_inner
    specs = [("transformer.embeddings.word_embeddings.weight", (V, h)),
             ("lm_head.weight", (V, h)), ("transformer.ln_f.weight", None)]
    for i in range(config.n_layer):
        q = f"transformer.layers.{i}."
        specs += [(q + "norm1.weight", None), (q + "norm2.weight", None),
                  (q + "mixer.Wqkv.weight", ((n_head + 2 * n_head_kv) * d, h)),
                  (q + "mixer.out_proj.weight", (h, n_head * d)),
                  (q + "mlp.fc1.weight", (2 * I, h)), (q + "mlp.fc2.weight", (h, I))]
    out = {}
    for name, size in specs:
        if size is None:
            out[name] = torch.ones(h, dtype=dtype, device=device)
            continue
        g = torch.Generator(device=device).manual_seed(_seed_for(name, seed))
        full = torch.empty(size, dtype=dtype, device=device)
        full.normal_(0.0, std, generator=g)
        if tp_world > 1:
            full = shard_state_dict_tp({name: full}, config, tp_world, tp_rank)[name].contiguous()
        out[name] = full
    return out
