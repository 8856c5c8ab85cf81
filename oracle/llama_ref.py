"""ORACLE (test infrastructure, never shipped): CPU restatement of HexGen-2's native Llama path.

Parity status: PINNED. tests/golden/make_golden.py runs the reference's own code
(hexgen/hexgen_core GPTLMHeadModel through hexgen2/model.py Engine.prefill/decode) on CPU and
commits its tokens, logits and KV bytes; tests/test_oracle_golden.py checks this restatement
against them.

What it restates (paths inside the HexGen-2 project):
  * HF -> native weight remap ........ hexgen/llama/load_model_parameters_utils/remap_state_dict.py:14-115
  * config mapping ................... hexgen/llama/llama_config_utils.py:39-67 + hexgen2/model.py:48-56
  * GPTModel / GPTLMHeadModel forward  hexgen/hexgen_core/models/gpt.py:363-417, :463-483
  * prenorm Block .................... hexgen/hexgen_core/modules/block.py:125-175
  * TorchRMSNorm ..................... hexgen/hexgen_core/modules/rms_norm.py:13-15
  * MHA forward (MHA and GQA branches) hexgen/hexgen_core/modules/mha.py:487-527, :539-573
  * _update_kv_cache ................. hexgen/hexgen_core/modules/mha.py:255-288
  * CrossAttention (CPU attention) ... hexgen/hexgen_core/modules/mha.py:209-244
  * GatedMlp ......................... hexgen/hexgen_core/modules/mlp.py:79-87
  * Engine.prefill / Engine.decode ... hexgen2/model.py:70-121
  * TP-shard concat of KV caches ..... hexgen/llama/tensor_parallel_dim_concat.py:9-21
Third-party arithmetic restated from its published algorithm (flash-attn 2.7.4.post1, git
5231d95fe13733fb534c01895f7ea88c6a6c7793, pinned by scripts/fabric/setup.sh:52-54):
  * RotaryEmbedding: inv_freq = 1/base^(arange(0,d,2)/d) in f32, cos/sin of outer(t, inv_freq)
    cached in the activation dtype, rotation evaluated in f32 and rounded (layers/rotary.py,
    ops/triton/rotary.py).
  * flash_attn_kvpacked_func numerics (attention="flash"): f32 scores and softmax, P rounded to
    the activation dtype before P.V, f32 accumulation, bottom-right causal alignment.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F


# ------------------------------------------------------------------------------- config
@dataclass
class LlamaShape:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    rms_norm_eps: float
    rope_theta: float = 10000.0

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @classmethod
    def from_hf(cls, cfg) -> "LlamaShape":
        """From a transformers LlamaConfig (or a dict with the same keys)."""
        get = (lambda k, d=None: cfg.get(k, d)) if isinstance(cfg, dict) else (
            lambda k, d=None: getattr(cfg, k, d))
        theta = get("rope_theta")
        if theta is None:
            params = get("rope_parameters") or {}
            theta = params.get("rope_theta", 10000.0)
        return cls(get("vocab_size"), get("hidden_size"), get("intermediate_size"),
                   get("num_hidden_layers"), get("num_attention_heads"),
                   get("num_key_value_heads") or get("num_attention_heads"),
                   float(get("rms_norm_eps")), float(theta))


# ------------------------------------------------------------------------------- weights
def remap_hf_to_native(state: dict, shape: LlamaShape) -> dict:
    """remap_state_dict.py:14-115 — HF names/layout to the native model's."""
    out = {}
    out["transformer.embeddings.word_embeddings.weight"] = state["model.embed_tokens.weight"]
    out["lm_head.weight"] = state["lm_head.weight"]
    out["transformer.ln_f.weight"] = state["model.norm.weight"]
    half = shape.head_dim // 2

    def inv_permute(w):  # '(h two d) n -> (h d two) n', d = head_dim / 2   (:88-93)
        h = w.shape[0] // (2 * half)
        return w.reshape(h, 2, half, w.shape[1]).transpose(1, 2).reshape(w.shape)

    for i in range(shape.num_layers):
        p = f"model.layers.{i}."
        q = f"transformer.layers.{i}."
        out[q + "norm1.weight"] = state[p + "input_layernorm.weight"]
        out[q + "norm2.weight"] = state[p + "post_attention_layernorm.weight"]
        out[q + "mixer.Wqkv.weight"] = torch.cat([
            inv_permute(state[p + "self_attn.q_proj.weight"]),
            inv_permute(state[p + "self_attn.k_proj.weight"]),
            state[p + "self_attn.v_proj.weight"]], dim=0)
        out[q + "mixer.out_proj.weight"] = state[p + "self_attn.o_proj.weight"]
        out[q + "mlp.fc1.weight"] = torch.cat([state[p + "mlp.up_proj.weight"],
                                              state[p + "mlp.gate_proj.weight"]], dim=0)
        out[q + "mlp.fc2.weight"] = state[p + "mlp.down_proj.weight"]
    return out


def random_native_state(shape: LlamaShape, seed: int, dtype=torch.float32, std=0.02,
                        layers=None) -> dict:
    """Seeded N(0, std) weights in native names (norm weights ones), generated on the CPU in
    f32 per tensor name and cast to `dtype`, so any consumer can regenerate them exactly."""
    import zlib
    layers = range(shape.num_layers) if layers is None else layers
    d, h, hq, hk = shape.head_dim, shape.hidden_size, shape.num_heads, shape.num_kv_heads

    def rnd(name, *size):
        g = torch.Generator().manual_seed((seed * 1000003 + zlib.crc32(name.encode())) & 0x7FFFFFFF)
        return (torch.randn(*size, generator=g) * std).to(dtype)

    out = {"transformer.embeddings.word_embeddings.weight": rnd("embed", shape.vocab_size, h),
           "lm_head.weight": rnd("lm_head", shape.vocab_size, h),
           "transformer.ln_f.weight": torch.ones(h, dtype=dtype)}
    for i in layers:
        q = f"transformer.layers.{i}."
        out[q + "norm1.weight"] = torch.ones(h, dtype=dtype)
        out[q + "norm2.weight"] = torch.ones(h, dtype=dtype)
        out[q + "mixer.Wqkv.weight"] = rnd(q + "Wqkv", (hq + 2 * hk) * d, h)
        out[q + "mixer.out_proj.weight"] = rnd(q + "out_proj", h, hq * d)
        out[q + "mlp.fc1.weight"] = rnd(q + "fc1", 2 * shape.intermediate_size, h)
        out[q + "mlp.fc2.weight"] = rnd(q + "fc2", h, shape.intermediate_size)
    return out


# ------------------------------------------------------------------------------- ops
def rms_norm(x, weight, eps):
    """rms_norm.py:13-15."""
    normalized = x.float() * torch.rsqrt(x.float().square().mean(-1, keepdim=True) + eps)
    return normalized.to(x.dtype) * weight


class Rotary:
    """flash_attn RotaryEmbedding (interleaved=True for the native Llama, mha.py:382-384)."""

    def __init__(self, dim: int, base: float, interleaved: bool = True):
        self.dim, self.base, self.interleaved = dim, float(base), interleaved
        self.inv_freq = 1.0 / (self.base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))

    def tables(self, seqlen: int, dtype):
        t = torch.arange(seqlen, dtype=torch.float32)
        freqs = torch.outer(t, self.inv_freq)
        return torch.cos(freqs).to(dtype), torch.sin(freqs).to(dtype)

    def apply(self, x, offset: int, dtype):
        """x: [B, S, H, D] -> rotated copy, f32 math, rounded to dtype."""
        s = x.shape[1]
        cos, sin = self.tables(offset + s, dtype)
        c = cos[offset:offset + s].float()[None, :, None, :]
        sn = sin[offset:offset + s].float()[None, :, None, :]
        xf = x.float()
        if self.interleaved:
            x0, x1 = xf[..., 0::2], xf[..., 1::2]
        else:
            x0, x1 = xf[..., : self.dim // 2], xf[..., self.dim // 2:]
        o0 = x0 * c - x1 * sn
        o1 = x0 * sn + x1 * c
        if self.interleaved:
            out = torch.stack((o0, o1), dim=-1).reshape(xf.shape)
        else:
            out = torch.cat((o0, o1), dim=-1)
        return out.to(dtype)


def cross_attention_torch(q, kv, causal, softmax_scale):
    """CrossAttention.forward, mha.py:209-244 (the reference's CPU attention)."""
    seqlen_q, seqlen_k = q.shape[1], kv.shape[1]
    if kv.shape[3] != q.shape[2]:
        kv = kv.repeat_interleave(q.shape[2] // kv.shape[3], dim=3)
    k, v = kv.unbind(dim=2)
    scale = softmax_scale or 1.0 / math.sqrt(q.shape[-1])
    scores = torch.einsum("bthd,bshd->bhts", q, k * scale)
    if causal:
        mask = torch.triu(torch.full((seqlen_q, seqlen_k), -10000.0), 1)
        scores = scores + mask.to(dtype=scores.dtype)
    attention = torch.softmax(scores, dim=-1, dtype=v.dtype)
    return torch.einsum("bhts,bshd->bthd", attention, v)


def flash_attention(q, kv, causal, softmax_scale):
    """flash_attn_kvpacked_func numerics: f32 scores/softmax, P rounded to the input dtype
    before P.V, f32 accumulation, bottom-right causal alignment, output rounded."""
    dtype = q.dtype
    seqlen_q, seqlen_k = q.shape[1], kv.shape[1]
    if kv.shape[3] != q.shape[2]:
        kv = kv.repeat_interleave(q.shape[2] // kv.shape[3], dim=3)
    k, v = kv.float().unbind(dim=2)
    scores = torch.einsum("bthd,bshd->bhts", q.float(), k) * softmax_scale
    if causal:
        qpos = torch.arange(seqlen_q)[:, None] + (seqlen_k - seqlen_q)
        keep = torch.arange(seqlen_k)[None, :] <= qpos
        scores = scores.masked_fill(~keep, float("-inf"))
    m = scores.amax(dim=-1, keepdim=True)
    p = torch.exp(scores - m)
    denom = p.sum(dim=-1, keepdim=True)
    p = p.to(dtype).float()
    out = torch.einsum("bhts,bshd->bthd", p, v) / denom.permute(0, 2, 1, 3)
    return out.to(dtype)


@dataclass
class CacheState:
    """hexgen2/model.py:12-20 (same field names)."""
    max_sequence_len: int
    max_batch_size: int = 1
    sequence_len_offset: int = 0
    batch_size_offset: int = 0
    key_value_memory_dict: dict = field(default_factory=dict)
    fused_ft_kernel: bool = False
    lengths_per_sample: object = None


# ------------------------------------------------------------------------------- model
class OracleModel:
    """GPTLMHeadModel forward for the native Llama configuration, on the CPU."""

    def __init__(self, shape: LlamaShape, native_state: dict, dtype=torch.float32,
                 attention: str = "torch"):
        self.shape, self.dtype, self.attention = shape, dtype, attention
        self.w = {k: v.to(dtype) for k, v in native_state.items()}
        self.rotary = Rotary(shape.head_dim, shape.rope_theta, interleaved=True)
        self.scale = shape.head_dim ** -0.5  # create_mixer_cls, gpt.py:72

    def _attn(self, q, kv, causal):
        if self.attention == "flash":
            return flash_attention(q, kv, causal, self.scale)
        return cross_attention_torch(q, kv, causal, self.scale)

    def _update_kv_cache(self, kv, params: CacheState, layer):
        """mha.py:255-288."""
        if layer not in params.key_value_memory_dict:
            params.key_value_memory_dict[layer] = torch.empty(
                params.max_batch_size, params.max_sequence_len, 2, kv.shape[-2], kv.shape[-1],
                dtype=kv.dtype)
        cache = params.key_value_memory_dict[layer]
        b0, b1 = params.batch_size_offset, params.batch_size_offset + kv.shape[0]
        s0, s1 = params.sequence_len_offset, params.sequence_len_offset + kv.shape[1]
        assert b1 <= cache.shape[0] and s1 <= cache.shape[1]
        cache[b0:b1, s0:s1, ...] = kv
        return cache[b0:b1, :s1, ...]

    def _mha(self, x, layer, params: CacheState | None):
        sh, w = self.shape, self.w
        d, hq, hk = sh.head_dim, sh.num_heads, sh.num_kv_heads
        qkv = F.linear(x, w[f"transformer.layers.{layer}.mixer.Wqkv.weight"])
        offset = 0 if params is None else params.sequence_len_offset
        q = qkv[..., : hq * d].reshape(*qkv.shape[:-1], hq, d)
        kv = qkv[..., hq * d:].reshape(*qkv.shape[:-1], 2, hk, d)
        q = self.rotary.apply(q, offset, self.dtype)
        k = self.rotary.apply(kv[:, :, 0], offset, self.dtype)
        kv = torch.stack((k, kv[:, :, 1]), dim=2)
        if params is None:
            ctx = self._attn(q, kv, True)
        else:
            kv = self._update_kv_cache(kv, params, layer)
            causal = params.sequence_len_offset == 0
            ctx = self._attn(q, kv, causal)
        return F.linear(ctx.reshape(*ctx.shape[:2], hq * d),
                        w[f"transformer.layers.{layer}.mixer.out_proj.weight"])

    def _mlp(self, x, layer):
        """mlp.py:79-87 (SwiGLU: fc1 rows are [up; gate])."""
        y = F.linear(x, self.w[f"transformer.layers.{layer}.mlp.fc1.weight"])
        y, gate = y.chunk(2, dim=-1)
        y = y * F.silu(gate)
        return F.linear(y, self.w[f"transformer.layers.{layer}.mlp.fc2.weight"])

    @torch.inference_mode()
    def forward(self, input_ids, params: CacheState | None = None, last_token_only=False):
        """gpt.py:363-417 + :463-483 (embeddings -> blocks -> ln_f -> lm_head)."""
        sh, w, eps = self.shape, self.w, self.shape.rms_norm_eps
        hidden = F.embedding(input_ids, w["transformer.embeddings.word_embeddings.weight"])
        residual = None
        for i in range(sh.num_layers):
            p = f"transformer.layers.{i}."
            residual = hidden + residual if residual is not None else hidden
            hidden = rms_norm(residual, w[p + "norm1.weight"], eps)
            hidden = self._mha(hidden, i, params)
            residual = hidden + residual
            hidden = rms_norm(residual, w[p + "norm2.weight"], eps)
            hidden = self._mlp(hidden, i)
        residual = hidden + residual
        hidden = rms_norm(residual, w["transformer.ln_f.weight"], eps)
        if last_token_only:
            hidden = hidden[:, -1]
        return F.linear(hidden, w["lm_head.weight"])

    # ------------------------------------------------------------ Engine flow (model.py:70-121)
    @torch.inference_mode()
    def prefill(self, input_ids, max_new_tokens):
        ids = torch.tensor([input_ids], dtype=torch.long)
        state = CacheState(len(input_ids) + max_new_tokens)
        logits = self.forward(ids, state, last_token_only=True)
        cache = {i: t[:, : len(input_ids)].contiguous()
                 for i, t in state.key_value_memory_dict.items()}
        return logits.argmax(-1), cache, logits

    @torch.inference_mode()
    def decode(self, first_token, cache, prompt_length, max_new_tokens, return_logits=False):
        token = first_token.reshape(1)
        generated = [int(token.item())]
        all_logits = []
        sh = self.shape
        if set(cache) != set(range(sh.num_layers)):
            raise ValueError("KV cache does not match the configured layer count")
        expected = (1, prompt_length, 2, sh.num_kv_heads, sh.head_dim)
        for value in cache.values():
            if tuple(value.shape) != expected or value.dtype != self.dtype:
                raise ValueError("KV cache shape/dtype does not match checkpoint and prompt")
        state = CacheState(prompt_length + max_new_tokens)
        state.sequence_len_offset = prompt_length
        for i, live in cache.items():
            full = torch.empty((1, state.max_sequence_len, *live.shape[2:]), dtype=self.dtype)
            full[:, :prompt_length].copy_(live)
            state.key_value_memory_dict[i] = full
        for _ in range(max_new_tokens - 1):
            logits = self.forward(token[:, None], state, last_token_only=True)
            all_logits.append(logits)
            state.sequence_len_offset += 1
            token = logits.argmax(-1)
            generated.append(int(token.item()))
        return (generated, all_logits) if return_logits else generated


class RaggedBatch:
    """Batched decode of requests with their own live lengths, for timing the reference
    algorithm on the host at a serving batch. The reference's Engine decodes one request at a
    time (model.py:85-121) and its legacy batching pads every cache to the longest
    (kv_cache_batch.py:4-29); here each request keeps its own cache and length, the projections
    run once for all B rows (F.linear over [B, h]) and attention runs per request over its own
    live rows, so the arithmetic is the reference's per-request decode step with the weight
    reads shared across the batch. Used only as the CPU baseline, never as a checker."""

    def __init__(self, model: OracleModel, caches: list[dict], lengths: list[int]):
        self.m, self.caches, self.lengths = model, caches, list(lengths)

    @torch.inference_mode()
    def step(self, tokens: torch.Tensor) -> torch.Tensor:
        """tokens [B] int64 -> logits [B, V]; every cache grows by one row."""
        m, sh, w, eps = self.m, self.m.shape, self.m.w, self.m.shape.rms_norm_eps
        d, hq, hk = sh.head_dim, sh.num_heads, sh.num_kv_heads
        B = tokens.numel()
        hidden = F.embedding(tokens.view(B, 1), w["transformer.embeddings.word_embeddings.weight"])
        residual = None
        for i in range(sh.num_layers):
            p = f"transformer.layers.{i}."
            residual = hidden + residual if residual is not None else hidden
            x = rms_norm(residual, w[p + "norm1.weight"], eps)
            qkv = F.linear(x, w[p + "mixer.Wqkv.weight"])  # [B, 1, (hq + 2hk) d]
            ctx = torch.empty(B, 1, hq * d, dtype=m.dtype)
            for b in range(B):
                L = self.lengths[b]
                q = qkv[b:b + 1, :, : hq * d].reshape(1, 1, hq, d)
                kv = qkv[b:b + 1, :, hq * d:].reshape(1, 1, 2, hk, d)
                q = m.rotary.apply(q, L, m.dtype)
                k = m.rotary.apply(kv[:, :, 0], L, m.dtype)
                cache = self.caches[b][i]
                cache[:, L, 0] = k[:, 0]
                cache[:, L, 1] = kv[:, 0, 1]
                ctx[b] = m._attn(q, cache[:, :L + 1], False).reshape(1, hq * d)
            hidden = F.linear(ctx, w[p + "mixer.out_proj.weight"])
            residual = hidden + residual
            x = rms_norm(residual, w[p + "norm2.weight"], eps)
            hidden = m._mlp(x, i)
        residual = hidden + residual
        x = rms_norm(residual, w["transformer.ln_f.weight"], eps)
        self.lengths = [L + 1 for L in self.lengths]
        return F.linear(x[:, -1], w["lm_head.weight"])


def load_hf_checkpoint(folder, dtype=torch.float32):
    """Reads a HF Llama safetensors checkpoint: (LlamaShape, native state dict)."""
    import json
    from pathlib import Path
    from safetensors.torch import load_file
    folder = Path(folder)
    cfg = json.loads((folder / "config.json").read_text())
    shape = LlamaShape.from_hf(cfg)
    state = {}
    for shard in sorted(folder.glob("*.safetensors")):
        state.update(load_file(str(shard), device="cpu"))
    return shape, remap_hf_to_native(state, shape)


def concat_kv_heads(shards: list[dict], dim: int = 3) -> dict:
    """hexgen/llama/tensor_parallel_dim_concat.py:9-21 (concat_dicts): the per-layer caches of
    the tensor-parallel shards, [B, S, 2, heads/tp, d] each, concatenated on the head dimension
    (dim 3) in rank order."""
    return {k: torch.cat([d[k] for d in shards], dim=dim) for k in shards[0]}
