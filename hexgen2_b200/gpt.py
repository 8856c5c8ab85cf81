"""Native Llama GPTLMHeadModel on the hexgen2_b200 sm_100a kernels.

Drop-in for the reference's native model (hexgen/hexgen_core/models/gpt.py:420-509 built with
the Llama configuration of hexgen/llama/llama_config_utils.py:39-67): same constructor
arguments, the same parameter names (so the reference's remapped state dicts load with
strict=True), the same forward signature and result type, and the same inference-cache
object (CacheState / InferenceParams fields). Tensor parallelism follows ParallelMHA /
ParallelGatedMlp / ParallelGPT2Embeddings (mha.py:576-735, mlp.py:90-118,
embedding.py:141-183) with NCCL all-reduce inside the process group.

The forward does not call the submodules one by one: it runs one fused plan per layer
    Wqkv GEMM -> rotary + KV-cache write -> attention -> out_proj GEMM (+ residual epilogue)
    -> RMSNorm -> fc1 GEMM (SwiGLU epilogue) -> fc2 GEMM (+ residual epilogue) -> RMSNorm
with the reference's rounding points (see the kernels), and only the last token's rows go
through the final norm and the LM head when last_token_only is set.
"""
from __future__ import annotations

from collections import namedtuple
from dataclasses import dataclass, field

import torch
import torch.distributed as dist
from torch import nn

from . import ops
from ._lib import HX_EPI_RESIDUAL, HX_EPI_SWIGLU

CausalLMOutput = namedtuple("CausalLMOutput", ["logits"])


@dataclass
class CacheState:
    """Inference cache (hexgen2/model.py:12-20; InferenceParams in
    hexgen/llama/inference_phases.py:20-40). key_value_memory_dict maps layer -> cache
    [max_batch_size, max_sequence_len, 2, n_heads_kv_local, head_dim]. When
    lengths_per_sample is an int32 CUDA tensor [batch] it gives each sequence's own offset
    (ragged batches); otherwise every sequence is at sequence_len_offset."""
    max_sequence_len: int
    max_batch_size: int = 1
    sequence_len_offset: int = 0
    batch_size_offset: int = 0
    key_value_memory_dict: dict = field(default_factory=dict)
    fused_ft_kernel: bool = False
    lengths_per_sample: object = None


InferenceParams = CacheState


def interleave_gated(w: torch.Tensor) -> torch.Tensor:
    """[up; gate] rows -> blocks of 16 [up16 | gate16] (the SwiGLU-epilogue layout)."""
    n = w.shape[0] // 2
    if n % 16:
        raise ValueError("GatedMlp hidden size must be a multiple of 16")
    up, gate = w[:n], w[n:]
    return torch.stack((up.reshape(n // 16, 16, -1), gate.reshape(n // 16, 16, -1)),
                       dim=1).reshape(w.shape).contiguous()


def deinterleave_gated(w: torch.Tensor) -> torch.Tensor:
    n = w.shape[0] // 2
    blocks = w.reshape(n // 16, 2, 16, -1)
    return torch.cat((blocks[:, 0].reshape(n, -1), blocks[:, 1].reshape(n, -1)), dim=0)


def _pg_size(pg):
    return 1 if pg is None else dist.get_world_size(pg)


def argmax_keys(values: torch.Tensor, global_index: torch.Tensor) -> torch.Tensor:
    """int64 keys whose maximum over tensor-parallel ranks is the greedy token of the whole
    vocabulary: the high 32 bits order the f32 values (sign-magnitude bits made monotone,
    -0.0 folded into +0.0), the low 32 bits hold 2^32 - 1 - index, so equal values resolve to
    the lowest vocabulary index, as torch.argmax over the gathered logits does."""
    bits = (values.float() + 0.0).view(torch.int32)
    ordered = torch.where(bits < 0, bits ^ 0x7FFFFFFF, bits).to(torch.int64)
    return ordered * 4294967296 + (4294967295 - global_index.to(torch.int64))


def key_index(key: torch.Tensor) -> torch.Tensor:
    """Vocabulary index carried by an argmax_keys key."""
    return 4294967295 - (key & 4294967295)


def _pg_rank(pg):
    return 0 if pg is None else dist.get_rank(pg)


class RMSNorm(nn.Module):
    """TorchRMSNorm (hexgen/hexgen_core/modules/rms_norm.py:6-15) on the fused kernel."""

    def __init__(self, hidden_size, eps=1e-6, device=None, dtype=None):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size, device=device, dtype=dtype))
        self.register_parameter("bias", None)
        self.eps = eps

    def forward(self, x):
        return ops.rmsnorm(x.reshape(-1, x.shape[-1]), self.weight, self.eps).view(x.shape)


class GPT2Embeddings(nn.Module):
    """embedding.py:12-51 (no position embeddings: n_positions = 0 for Llama)."""

    def __init__(self, embed_dim, vocab_size, max_position_embeddings=0, padding_idx=None,
                 device=None, dtype=None):
        super().__init__()
        self.word_embeddings = nn.Embedding(vocab_size, embed_dim, padding_idx=padding_idx,
                                            device=device, dtype=dtype)
        self.max_position_embeddings = 0

    def forward(self, input_ids, position_ids=None):
        return ops.embedding(input_ids.reshape(-1), self.word_embeddings.weight).view(
            *input_ids.shape, -1)


class ParallelGPT2Embeddings(nn.Module):
    """Vocab-parallel embedding + all-reduce (embedding.py:96-124, :141-183)."""

    def __init__(self, embed_dim, vocab_size, max_position_embeddings, process_group,
                 padding_idx=None, sequence_parallel=False, device=None, dtype=None):
        super().__init__()
        world = _pg_size(process_group)
        if vocab_size % world:
            raise ValueError(f"num_embeddings ({vocab_size}) must be divisible by world_size ({world})")
        self.process_group = process_group
        self.sequence_parallel = False
        self.word_embeddings = nn.Embedding(vocab_size // world, embed_dim, device=device, dtype=dtype)
        self.max_position_embeddings = 0

    def forward(self, input_ids, position_ids=None, combine_batch_seqlen_dim=False):
        rank = _pg_rank(self.process_group)
        rows = self.word_embeddings.weight.shape[0]
        out = ops.embedding(input_ids.reshape(-1), self.word_embeddings.weight, rank * rows)
        if _pg_size(self.process_group) > 1:
            dist.all_reduce(out, group=self.process_group)
        return out.view(*input_ids.shape, -1)


class MHA(nn.Module):
    """Self-attention mixer of the native Llama (mha.py:344-573): fused Wqkv, interleaved
    rotary, KV-cache update, causal prefill / cached decode attention, out_proj. With a
    process_group it is ParallelMHA (mha.py:576-735): heads split across ranks."""

    def __init__(self, embed_dim, num_heads, num_heads_kv=None, process_group=None,
                 qkv_proj_bias=False, out_proj_bias=False, dropout=0.0, softmax_scale=None,
                 causal=True, layer_idx=None, rotary_emb_dim=0, rotary_emb_base=10000.0,
                 rotary_emb_interleaved=True, device=None, dtype=None, **unused):
        super().__init__()
        if qkv_proj_bias or out_proj_bias:
            raise ValueError("the native Llama attention has no biases")
        self.embed_dim, self.layer_idx, self.causal = embed_dim, layer_idx, causal
        self.process_group = process_group
        world = _pg_size(process_group)
        self.num_heads = num_heads
        self.num_heads_kv = num_heads_kv or num_heads
        if self.num_heads % self.num_heads_kv or self.num_heads_kv % world or embed_dim % num_heads:
            raise ValueError("head counts must divide evenly (and by the TP size)")
        self.head_dim = embed_dim // num_heads
        self.num_heads_per_rank = num_heads // world
        self.num_heads_kv_per_rank = self.num_heads_kv // world
        self.softmax_scale = softmax_scale or self.head_dim ** -0.5
        self.rotary_emb_dim = rotary_emb_dim
        self.rotary_emb_base = float(rotary_emb_base)
        self.rotary_emb_interleaved = rotary_emb_interleaved
        qkv_dim = self.head_dim * (self.num_heads_per_rank + 2 * self.num_heads_kv_per_rank)
        self.Wqkv = nn.Linear(embed_dim, qkv_dim, bias=False, device=device, dtype=dtype)
        self.out_proj = nn.Linear(self.num_heads_per_rank * self.head_dim, embed_dim, bias=False,
                                  device=device, dtype=dtype)


class GatedMlp(nn.Module):
    """SwiGLU MLP (mlp.py:63-87); with a process_group it is ParallelGatedMlp (mlp.py:90-118).
    fc1.weight is held interleaved in blocks of 16 rows ([up16 | gate16]) so the fc1 GEMM
    epilogue can form up * silu(gate); state dicts use the reference's [up; gate] layout."""

    def __init__(self, in_features, hidden_features=None, process_group=None, out_features=None,
                 device=None, dtype=None, multiple_of=256, **unused):
        super().__init__()
        out_features = out_features or in_features
        hidden = hidden_features or int(8 * in_features / 3)
        hidden = (hidden + multiple_of - 1) // multiple_of * multiple_of if hidden_features is None else hidden
        world = _pg_size(process_group)
        if hidden % world:
            raise ValueError("MLP hidden size must divide by the TP size")
        self.process_group = process_group
        self.hidden_local = hidden // world
        self.fc1 = nn.Linear(in_features, 2 * self.hidden_local, bias=False, device=device, dtype=dtype)
        self.fc2 = nn.Linear(self.hidden_local, out_features, bias=False, device=device, dtype=dtype)
        self._register_state_dict_hook(GatedMlp._export_hook)
        self._register_load_state_dict_pre_hook(GatedMlp._import_hook)

    @staticmethod
    def _export_hook(module, state, prefix, local_metadata):
        key = prefix + "fc1.weight"
        if key in state:
            state[key] = deinterleave_gated(state[key])
        return state

    @staticmethod
    def _import_hook(state, prefix, *args):
        key = prefix + "fc1.weight"
        if key in state:
            state[key] = interleave_gated(state[key])


class Block(nn.Module):
    """Prenorm block (block.py:37-175): Add -> Norm -> Mixer -> Add -> Norm -> MLP."""

    def __init__(self, dim, mixer, mlp, eps, device=None, dtype=None):
        super().__init__()
        self.mixer = mixer
        self.norm1 = RMSNorm(dim, eps=eps, device=device, dtype=dtype)
        self.mlp = mlp
        self.norm2 = RMSNorm(dim, eps=eps, device=device, dtype=dtype)


def _cfg(config, *names, default=None):
    for n in names:
        v = getattr(config, n, None)
        if v is not None:
            return v
    return default


class GPTModel(nn.Module):
    """gpt.py:289-417 for the Llama configuration (RMSNorm, SwiGLU, rotary, no biases)."""

    def __init__(self, config, process_group=None, device=None, dtype=None):
        super().__init__()
        self.process_group = process_group
        hidden = _cfg(config, "n_embd", "hidden_size")
        n_head = _cfg(config, "n_head", "num_attention_heads")
        n_head_kv = _cfg(config, "n_head_kv", "num_key_value_heads", default=n_head)
        n_layer = _cfg(config, "n_layer", "num_hidden_layers")
        vocab = _cfg(config, "vocab_size")
        pad = getattr(config, "pad_vocab_size_multiple", 1) or 1
        vocab = (vocab + pad - 1) // pad * pad
        eps = _cfg(config, "layer_norm_epsilon", "rms_norm_eps", default=1e-6)
        inner = _cfg(config, "n_inner", "intermediate_size")
        head_dim = hidden // n_head
        rot_dim = int(_cfg(config, "rotary_emb_fraction", default=1.0) * head_dim)
        if rot_dim != head_dim:
            raise ValueError("the native Llama path rotates the full head dimension")
        if process_group is None:
            self.embeddings = GPT2Embeddings(hidden, vocab, device=device, dtype=dtype)
        else:
            self.embeddings = ParallelGPT2Embeddings(hidden, vocab, 0, process_group,
                                                     device=device, dtype=dtype)
        self.layers = nn.ModuleList()
        for i in range(n_layer):
            mixer = MHA(hidden, n_head, n_head_kv, process_group=process_group, layer_idx=i,
                        rotary_emb_dim=rot_dim,
                        rotary_emb_base=_cfg(config, "rotary_emb_base", default=10000.0),
                        rotary_emb_interleaved=bool(_cfg(config, "rotary_emb_interleaved", default=True)),
                        device=device, dtype=dtype)
            mlp = GatedMlp(hidden, inner, process_group=process_group, device=device, dtype=dtype)
            self.layers.append(Block(hidden, mixer, mlp, eps, device=device, dtype=dtype))
        self.ln_f = RMSNorm(hidden, eps=eps, device=device, dtype=dtype)


class GPTLMHeadModel(nn.Module):
    """gpt.py:420-509: GPTModel + untied LM head; forward(input_ids, position_ids=None,
    inference_params=None, last_token_only=False) -> CausalLMOutput(logits)."""

    def __init__(self, config, process_group=None, device=None, dtype=None):
        super().__init__()
        self.config = config
        self.process_group = process_group
        self.transformer = GPTModel(config, process_group=process_group, device=device, dtype=dtype)
        hidden = _cfg(config, "n_embd", "hidden_size")
        vocab = self.transformer.embeddings.word_embeddings.weight.shape[0]
        self.lm_head = nn.Linear(hidden, vocab, bias=False, device=device, dtype=dtype)
        m0 = self.transformer.layers[0].mixer
        self.n_layer = len(self.transformer.layers)
        self.hidden = hidden
        self.hq, self.hk, self.head_dim = m0.num_heads_per_rank, m0.num_heads_kv_per_rank, m0.head_dim
        self.scale = m0.softmax_scale
        self.eps = self.transformer.ln_f.eps
        self.tp = _pg_size(process_group)
        self._rope: dict = {}

    # ------------------------------------------------------------------ helpers
    def rope_tables(self, length: int, device, dtype):
        """cos/sin [rows, d/2] in the activation dtype, computed like flash_attn's
        RotaryEmbedding._update_cos_sin_cache (f32 outer product, cos/sin, cast)."""
        key = (device, dtype)
        tab = self._rope.get(key)
        if tab is None or tab[0].shape[0] < length:
            rows = max(length, 4096)
            m0 = self.transformer.layers[0].mixer
            d = m0.rotary_emb_dim
            inv_freq = 1.0 / (m0.rotary_emb_base ** (torch.arange(0, d, 2, device=device,
                                                                   dtype=torch.float32) / d))
            t = torch.arange(rows, device=device, dtype=torch.float32)
            freqs = torch.outer(t, inv_freq)
            tab = (torch.cos(freqs).to(dtype).contiguous(), torch.sin(freqs).to(dtype).contiguous())
            self._rope[key] = tab
        return tab

    def allocate_inference_cache(self, batch_size, max_seqlen, dtype=None, device=None):
        """One tensor for all layers; returns {layer: view [B, S, 2, hkv_local, d]}."""
        w = self.lm_head.weight
        big = torch.empty(self.n_layer, batch_size, max_seqlen, 2, self.hk, self.head_dim,
                          dtype=dtype or w.dtype, device=device or w.device)
        return {i: big[i] for i in range(self.n_layer)}

    def _all_reduce(self, t):
        if self.tp > 1:
            dist.all_reduce(t, group=self.process_group)

    # ------------------------------------------------------------------ forward
    @torch.inference_mode()
    def forward(self, input_ids, position_ids=None, inference_params=None, last_token_only=False,
                gather_logits=True):
        """gpt.py:463-483. With tensor parallelism the LM head is vocab-parallel; its logits are
        all-gathered into [.., vocab] as in the reference (gpt.py:479-481) unless gather_logits
        is False, in which case this rank's vocabulary slice is returned (next_tokens() uses
        that to pick the greedy token without gathering the logits)."""
        if input_ids.dim() != 2:
            raise ValueError("input_ids must be [batch, seqlen]")
        B, S = input_ids.shape
        w_emb = self.transformer.embeddings.word_embeddings.weight
        device, dtype = w_emb.device, w_emb.dtype
        h, hq, hk, d = self.hidden, self.hq, self.hk, self.head_dim
        params = inference_params
        if params is None:
            params = CacheState(max_sequence_len=S, max_batch_size=B)
        caches = params.key_value_memory_dict
        if any(i not in caches for i in range(self.n_layer)):
            fresh = self.allocate_inference_cache(params.max_batch_size, params.max_sequence_len,
                                                  dtype=dtype, device=device)
            for i in range(self.n_layer):
                caches.setdefault(i, fresh[i])
        b0 = params.batch_size_offset
        if isinstance(params.lengths_per_sample, torch.Tensor):
            pos = params.lengths_per_sample[b0:b0 + B].to(device=device, dtype=torch.int32)
            max_pos = int(params.max_sequence_len)
        else:
            pos = torch.full((B,), params.sequence_len_offset, dtype=torch.int32, device=device)
            max_pos = params.sequence_len_offset + S
        decode = S == 1 and (isinstance(params.lengths_per_sample, torch.Tensor)
                             or params.sequence_len_offset > 0)
        causal = isinstance(params.lengths_per_sample, torch.Tensor) or params.sequence_len_offset == 0
        cos, sin = self.rope_tables(max(max_pos, params.max_sequence_len), device, dtype)
        ids = input_ids.reshape(-1).to(device=device, dtype=torch.long).contiguous()
        rows = B * S
        residual = torch.empty(rows, h, dtype=dtype, device=device)
        normed = torch.empty(rows, h, dtype=dtype, device=device)
        layers = self.transformer.layers
        if self.tp == 1:
            ops.embed_rmsnorm(ids, w_emb, layers[0].norm1.weight, self.eps, residual, normed)
        else:
            emb = self.transformer.embeddings(ids.view(B, S)).view(rows, h)
            ops.rmsnorm(emb, layers[0].norm1.weight, self.eps, residual_out=residual, out=normed)
        seqlens = pos + 1 if decode else None
        for i, layer in enumerate(layers):
            mixer, mlp = layer.mixer, layer.mlp
            cache = caches[i]
            if dtype != torch.float32 and mixer.rotary_emb_interleaved:
                q = ops.gemm_qkv_rotary(normed, mixer.Wqkv.weight, S, hq, hk, d, pos, cos, sin,
                                        cache, batch_offset=b0).view(B, S, hq, d)
            else:
                qkv = ops.gemm(normed, mixer.Wqkv.weight)
                q = ops.rotary_cache_write(qkv, B, S, hq, hk, d, pos, cos, sin, cache,
                                           batch_offset=b0,
                                           interleaved=mixer.rotary_emb_interleaved)
            if decode:
                cview = cache[b0:b0 + B]
                ctx = ops.decode_attention(q.view(B, hq, d), cview, seqlens, hk, max_pos,
                                           self.scale)
            else:
                ctx = ops.prefill_attention(q, cache, pos, hk, self.scale, causal=causal,
                                            batch_offset=b0)
            ctx = ctx.view(rows, hq * d)
            if self.tp == 1:
                ops.gemm(ctx, mixer.out_proj.weight, HX_EPI_RESIDUAL, residual=residual, out=residual)
                ops.rmsnorm(residual, layer.norm2.weight, self.eps, out=normed)
            else:
                part = ops.gemm(ctx, mixer.out_proj.weight)
                self._all_reduce(part)
                ops.rmsnorm(part, layer.norm2.weight, self.eps, add=residual,
                            residual_out=residual, out=normed)
            act = ops.gemm(normed, mlp.fc1.weight, HX_EPI_SWIGLU)
            nxt = layers[i + 1].norm1.weight if i + 1 < len(layers) else None
            if self.tp == 1:
                ops.gemm(act, mlp.fc2.weight, HX_EPI_RESIDUAL, residual=residual, out=residual)
                if nxt is not None:
                    ops.rmsnorm(residual, nxt, self.eps, out=normed)
            else:
                part = ops.gemm(act, mlp.fc2.weight)
                self._all_reduce(part)
                if nxt is not None:
                    ops.rmsnorm(part, nxt, self.eps, add=residual, residual_out=residual, out=normed)
                else:
                    ops.rmsnorm(part, self.transformer.ln_f.weight, self.eps, add=residual,
                                residual_out=residual, out=normed)
        # Final norm (gpt.py:388-397) on the rows the LM head needs. With TP the last layer's
        # fused add + norm already applied ln_f to every row.
        if self.tp > 1:
            hfin = normed.view(B, S, h)[:, -1] if last_token_only else normed
        elif last_token_only:
            last = residual.view(B, S, h)[:, -1]
            hfin = ops.rmsnorm(last, self.transformer.ln_f.weight, self.eps, rows=B,
                               in_stride=S * h)
        else:
            hfin = ops.rmsnorm(residual, self.transformer.ln_f.weight, self.eps)
        logits = ops.gemm(hfin, self.lm_head.weight)
        if self.tp > 1 and gather_logits:
            parts = [torch.empty_like(logits) for _ in range(self.tp)]
            dist.all_gather(parts, logits, group=self.process_group)
            logits = torch.cat(parts, dim=-1)
        if not last_token_only:
            logits = logits.view(B, S, -1)
        return CausalLMOutput(logits=logits)

    @torch.inference_mode()
    def prefill_packed(self, input_ids, lengths, caches, slots, greedy=True, out=None):
        """Prefill of several prompts in ONE pass over their concatenated rows: input_ids is a
        flat int64 CUDA tensor of sum(lengths) tokens, prompt i of lengths[i] tokens goes to
        batch row slots[i] of `caches` ({layer: [B, capacity, 2, hkv, d]}, positions 0..L-1).
        Every projection, norm and residual add runs once over all rows (GEMM M = sum of the
        prompt lengths, which fills the GPU where a single prompt's rows do not); the Wqkv GEMM's
        epilogue rotates and writes every prompt's rows to its own cache row, and the causal
        attention of all prompts runs in one launch. Equals forward() of each prompt alone,
        logit for logit up to the summation order of the projections. Returns the greedy next token of every prompt (int64 [n]; TP:
        one all-reduce of keys, as next_tokens) or, with greedy=False, the last-token logits
        [n, vocab] (gathered across TP ranks)."""
        n = len(lengths)
        if n == 0 or len(slots) != n or any(L <= 0 for L in lengths):
            raise ValueError("prefill_packed needs one slot and a positive length per prompt")
        T = int(sum(lengths))
        if input_ids.dim() != 1 or input_ids.numel() != T:
            raise ValueError("input_ids must be the flat concatenation of the prompts")
        w_emb = self.transformer.embeddings.word_embeddings.weight
        device, dtype = w_emb.device, w_emb.dtype
        h, hq, hk, d = self.hidden, self.hq, self.hk, self.head_dim
        cap = caches[0].shape[1]
        if max(lengths) > cap:
            raise ValueError(f"a prompt of {max(lengths)} tokens exceeds the cache capacity {cap}")
        cos, sin = self.rope_tables(cap, device, dtype)
        ids = input_ids.to(device=device, dtype=torch.long)
        zero = torch.zeros(1, dtype=torch.int32, device=device)
        offs = [0]
        for L in lengths:
            offs.append(offs[-1] + L)
        residual = torch.empty(T, h, dtype=dtype, device=device)
        normed = torch.empty(T, h, dtype=dtype, device=device)
        q = torch.empty(T, hq, d, dtype=dtype, device=device)
        ctx = torch.empty(T, hq, d, dtype=dtype, device=device)
        layers = self.transformer.layers
        meta = ops.varlen_meta(lengths, slots, device)
        if self.tp == 1:
            ops.embed_rmsnorm(ids, w_emb, layers[0].norm1.weight, self.eps, residual, normed)
        else:
            emb = self.transformer.embeddings(ids.view(1, T)).view(T, h)
            ops.rmsnorm(emb, layers[0].norm1.weight, self.eps, residual_out=residual, out=normed)
        for i, layer in enumerate(layers):
            mixer, mlp = layer.mixer, layer.mlp
            cache = caches[i]
            if dtype != torch.float32 and mixer.rotary_emb_interleaved:
                # Rotary + KV-cache write of every prompt in the Wqkv GEMM's epilogue.
                ops.gemm_qkv_rotary_varlen(normed, mixer.Wqkv.weight, lengths, slots, hq, hk, d,
                                           cos, sin, cache, q, meta=meta)
            else:
                qkv = ops.gemm(normed, mixer.Wqkv.weight)
                for b in range(n):
                    o, L = offs[b], lengths[b]
                    ops.rotary_cache_write(qkv[o:o + L], 1, L, hq, hk, d, zero, cos, sin, cache,
                                           q_out=q[o:o + L].view(1, L, hq, d),
                                           batch_offset=slots[b],
                                           interleaved=mixer.rotary_emb_interleaved)
            # All prompts' causal attention in one launch (one grid over heads x 128-query
            # blocks of every prompt); prompt by prompt where that kernel does not apply.
            if not ops.prefill_attention_varlen(q, cache, lengths, slots, hk, self.scale, ctx,
                                                meta=meta):
                for b in range(n):
                    o, L = offs[b], lengths[b]
                    ops.prefill_attention(q[o:o + L].view(1, L, hq, d), cache, zero, hk,
                                          self.scale, causal=True,
                                          out=ctx[o:o + L].view(1, L, hq, d), batch_offset=slots[b])
            c2 = ctx.view(T, hq * d)
            if self.tp == 1:
                ops.gemm(c2, mixer.out_proj.weight, HX_EPI_RESIDUAL, residual=residual, out=residual)
                ops.rmsnorm(residual, layer.norm2.weight, self.eps, out=normed)
            else:
                part = ops.gemm(c2, mixer.out_proj.weight)
                self._all_reduce(part)
                ops.rmsnorm(part, layer.norm2.weight, self.eps, add=residual,
                            residual_out=residual, out=normed)
            act = ops.gemm(normed, mlp.fc1.weight, HX_EPI_SWIGLU)
            nxt = layers[i + 1].norm1.weight if i + 1 < len(layers) else None
            if self.tp == 1:
                ops.gemm(act, mlp.fc2.weight, HX_EPI_RESIDUAL, residual=residual, out=residual)
                if nxt is not None:
                    ops.rmsnorm(residual, nxt, self.eps, out=normed)
            else:
                part = ops.gemm(act, mlp.fc2.weight)
                self._all_reduce(part)
                ops.rmsnorm(part, nxt if nxt is not None else self.transformer.ln_f.weight,
                            self.eps, add=residual, residual_out=residual, out=normed)
        last = torch.tensor([o - 1 for o in offs[1:]], dtype=torch.long, device=device)
        if self.tp > 1:
            hfin = normed.index_select(0, last)
        else:
            hfin = ops.rmsnorm(residual.index_select(0, last), self.transformer.ln_f.weight, self.eps)
        logits = ops.gemm(hfin, self.lm_head.weight)
        if greedy:
            if self.tp == 1:
                return ops.argmax(logits, out=out)
            return self._tp_argmax(logits, out)
        if self.tp > 1:
            parts = [torch.empty_like(logits) for _ in range(self.tp)]
            dist.all_gather(parts, logits, group=self.process_group)
            logits = torch.cat(parts, dim=-1)
        return logits

    @torch.inference_mode()
    def next_tokens(self, input_ids, inference_params=None, out=None):
        """Greedy next token of every sequence: argmax of forward(..., last_token_only=True)
        with torch.argmax's tie rule (lowest vocabulary index). Returns int64 [batch].

        With tensor parallelism each rank takes the argmax of its own vocabulary slice and the
        ranks agree on the winner with ONE all-reduce(MAX) of one int64 key per sequence: the
        high 32 bits order the logit value (its f32 bit pattern mapped to a signed integer of the
        same order), the low 32 bits are (2^32 - 1 - global index), so equal values resolve to
        the lowest index, as on the gathered logits. This replaces the all-gather of
        [batch, vocab / TP] logits (gpt.py:479-481) on the decode path."""
        logits = self.forward(input_ids, inference_params=inference_params, last_token_only=True,
                              gather_logits=False).logits
        if self.tp == 1:
            return ops.argmax(logits, out=out)
        return self._tp_argmax(logits, out)

    def _tp_argmax(self, local_logits, out=None):
        rows, vloc = local_logits.shape
        idx = ops.argmax(local_logits)
        val = local_logits.gather(1, idx.view(rows, 1)).view(rows)
        key = argmax_keys(val, idx + _pg_rank(self.process_group) * vloc)
        dist.all_reduce(key, op=dist.ReduceOp.MAX, group=self.process_group)
        win = key_index(key)
        if out is None:
            return win
        out.copy_(win)
        return out
