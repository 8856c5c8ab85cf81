"""Engine: the prefill/decode API of hexgen2/model.py:23-124 on the B200 kernels.

Same constructor, attributes and methods as the reference's native engine:
    Engine(model_dir, engine="native", device="cuda", dtype="float16")
    .config (HF LlamaConfig), .identity, .kind, .model
    .prefill(input_ids, max_new_tokens) -> (LongTensor[1], {layer: Tensor[1, L, 2, hkv, d]}, logits[1, V])
    .decode(first_token, cache, prompt_length, max_new_tokens, on_token=None) -> list[int]
    .synchronize()
and the same ValueError conditions. Differences that do not change results:
  * prefill packs every layer's live cache rows with one gather kernel into one buffer that the
    caller owns; the returned per-layer tensors are contiguous views of it;
  * decode re-expands the received live rows into one all-layer cache with one scatter kernel;
  * greedy argmax runs on the GPU (hx_argmax, torch.argmax tie-breaking).
Also: Engine.from_config(...) builds a seeded random-init model of any Llama shape on the
device (no checkpoint files), and decode_batch() runs ragged batches with per-sequence
lengths (continuous-batching building block). Engine(..., engine="hf-reference") is the
reference's validation engine (transformers' eager LlamaForCausalLM, prefill / decode only).
"""
from __future__ import annotations

import torch

from . import ops
from .checkpoint import (llama_config_to_gpt2_config, load_safetensors_dir, model_identity,
                         random_native_state, remap_state_dict_hf_llama, shard_state_dict_tp)
from .gpt import CacheState, GPTLMHeadModel


# Packed prefill passes: at most this many tokens (GEMM rows) and prompts per pass. 8192 rows
# fill every CTA pair of the projection GEMMs; the cap on prompts bounds the cache slots a
# prefill-only rank needs.
PREFILL_TOKENS = 8192
PREFILL_PROMPTS = 16


def _check_device(device: torch.device):
    if device.type != "cuda" or not torch.cuda.is_available():
        raise ValueError("Native HexGen-2 on B200 requires CUDA; the CPU reference lives in the oracle")
    major, minor = torch.cuda.get_device_capability(device)
    if (major, minor) != (10, 0):
        raise ValueError(f"hexgen2_b200 kernels are built for sm_100a (B200); got sm_{major}{minor}")


class Engine:
    def __init__(self, model_dir, engine="native", device="cuda", dtype="float16",
                 process_group=None):
        from transformers import LlamaConfig

        self.device, self.dtype = torch.device(device), getattr(torch, dtype)
        self.config = LlamaConfig.from_pretrained(model_dir, local_files_only=True)
        self.identity = model_identity(model_dir)
        scaling = getattr(self.config, "rope_scaling", None)
        if self.config.model_type != "llama" or (
                scaling is not None and scaling.get("rope_type", "default") != "default"):
            raise ValueError("This baseline supports Llama architecture without RoPE scaling")
        if engine == "hf-reference":
            # The reference's validation engine (hexgen2/model.py:32-37): transformers' eager
            # LlamaForCausalLM on any device, chosen explicitly by the caller. It runs none of
            # this package's kernels, and the native engine never falls back to it.
            from transformers import LlamaForCausalLM
            self.kind = engine
            self.model = LlamaForCausalLM.from_pretrained(
                model_dir, local_files_only=True, dtype=self.dtype, use_safetensors=True,
                attn_implementation="eager").to(self.device).eval()
            c = self.config
            self.num_layers, self.kv_heads = c.num_hidden_layers, c.num_key_value_heads
            self.head_dim = c.hidden_size // c.num_attention_heads
            return
        if engine != "native":
            raise ValueError(f"unknown engine {engine!r}: 'native' or 'hf-reference'")
        self.kind = engine
        _check_device(self.device)
        if self.device.index is not None:
            torch.cuda.set_device(self.device)
        gconfig = llama_config_to_gpt2_config(self.config)
        self.process_group = process_group
        state = remap_state_dict_hf_llama(load_safetensors_dir(model_dir), gconfig)
        if process_group is not None:
            state = shard_state_dict_tp(state, gconfig, torch.distributed.get_world_size(process_group),
                                        torch.distributed.get_rank(process_group))
        self.model = GPTLMHeadModel(gconfig, process_group=process_group, device=self.device,
                                    dtype=self.dtype).eval()
        # Strict loading prevents accidental use of uninitialised weights.
        self.model.load_state_dict(state, strict=True)
        self._post_init()

    @classmethod
    def from_config(cls, llama_config: dict, dtype="bfloat16", device="cuda", seed=0,
                    process_group=None):
        """Random-init model of the given Llama shape (weights N(0, 0.02), seeded per tensor
        name, generated on the device; every TP layout sees the same underlying weights)."""
        from transformers import LlamaConfig

        self = cls.__new__(cls)
        self.device, self.dtype = torch.device(device), getattr(torch, dtype)
        _check_device(self.device)
        self.config = LlamaConfig(**llama_config)
        self.identity = {"random_init_seed": seed}
        self.kind = "native"
        self.process_group = process_group
        gconfig = llama_config_to_gpt2_config(self.config)
        world = 1 if process_group is None else torch.distributed.get_world_size(process_group)
        rank = 0 if process_group is None else torch.distributed.get_rank(process_group)
        with torch.device("meta"):
            model = GPTLMHeadModel(gconfig, process_group=process_group, dtype=self.dtype)
        state = random_native_state(gconfig, seed=seed, dtype=self.dtype, device=self.device,
                                    tp_world=world, tp_rank=rank)
        model.load_state_dict(state, strict=True, assign=True)
        self.model = model.eval()
        self.model._rope = {}
        self._post_init()
        return self

    def _post_init(self):
        m = self.model
        self.num_layers = m.n_layer
        self.kv_heads = m.hk
        self.head_dim = m.head_dim
        self.row_bytes = 2 * m.hk * m.head_dim * torch.empty((), dtype=self.dtype).element_size()

    # ------------------------------------------------------------------ prefill / decode
    def _native_only(self, what: str):
        if self.kind != "native":
            raise ValueError(f"{what} needs the native engine (this one is {self.kind!r})")

    @torch.inference_mode()
    def prefill(self, input_ids, max_new_tokens):
        if self.kind == "hf-reference":
            return self._hf_prefill(input_ids)
        ids = torch.tensor([input_ids], dtype=torch.long, device=self.device)
        L = len(input_ids)
        state = CacheState(L + max_new_tokens)
        logits = self.model(ids, inference_params=state, last_token_only=True).logits
        # The returned cache holds the prompt's L written rows of every layer; the
        # max_new_tokens rows reserved for decoding stay behind.
        cache = self.pack_live(state.key_value_memory_dict, [L])[0]
        return ops.argmax(logits), cache, logits

    def pack_live(self, caches: dict, lengths: list[int], batch_rows=None):
        """Gathers rows [0, L_b) of cache slot b of every layer into one buffer per request.
        Returns a list (one per request) of {layer: [1, L_b, 2, hkv, d]} contiguous views."""
        self._native_only("pack_live")
        n = self.num_layers
        big0 = caches[0]
        layer_stride = (caches[1].data_ptr() - big0.data_ptr()) if n > 1 else 0
        uniform = n == 1 or all(caches[i].data_ptr() == big0.data_ptr() + i * layer_stride
                                for i in range(n))
        if not uniform:
            raise ValueError("pack_live expects the engine's single all-layer cache")
        rows = list(range(len(lengths))) if batch_rows is None else batch_rows
        elem = big0.element_size()
        total = sum(n * L for L in lengths)
        packed = torch.empty(total * self.row_bytes, dtype=torch.uint8, device=self.device)
        offs, o = [], 0
        for L in lengths:
            offs.append(o)
            o += n * L * self.row_bytes
        src = torch.tensor([big0.data_ptr() + r * big0.stride(0) * elem for r in rows],
                           dtype=torch.int64, device=self.device)
        live = torch.tensor(lengths, dtype=torch.int64, device=self.device)
        dst_off = torch.tensor(offs, dtype=torch.int64, device=self.device)
        ops.kv_pack(src, live, dst_off, n, layer_stride, big0.stride(1) * elem, self.row_bytes,
                    max(lengths), packed)
        out = []
        for L, off in zip(lengths, offs):
            view = packed[off:off + n * L * self.row_bytes].view(self.dtype).view(
                n, 1, L, 2, self.kv_heads, self.head_dim)
            out.append({i: view[i] for i in range(n)})
        return out

    def unpack_live(self, live_caches: list[dict], lengths: list[int], capacity: int):
        """Scatter received live caches (one dict per request) into a fresh all-layer cache
        [layers, B, capacity, 2, hkv, d]; returns {layer: [B, capacity, 2, hkv, d]}."""
        n, B = self.num_layers, len(live_caches)
        big = torch.empty(n, B, capacity, 2, self.kv_heads, self.head_dim, dtype=self.dtype,
                          device=self.device)
        elem = big.element_size()
        srcs, dsts, lens = [], [], []
        for b, (cache, L) in enumerate(zip(live_caches, lengths)):
            for i in range(n):
                t = cache[i]
                if not t.is_contiguous():
                    t = t.contiguous()
                if t.device != self.device:
                    t = t.to(self.device)
                    cache[i] = t
                srcs.append(t.data_ptr())
                dsts.append(big[i, b].data_ptr())
                lens.append(L)
        base = min(srcs)
        ops.kv_unpack(base, torch.tensor([s - base for s in srcs], dtype=torch.int64, device=self.device),
                      torch.tensor(lens, dtype=torch.int64, device=self.device),
                      torch.tensor(dsts, dtype=torch.int64, device=self.device), 1, 0,
                      big.stride(2) * elem, self.row_bytes, max(lengths))
        return {i: big[i] for i in range(n)}

    def _hf_prefill(self, input_ids):
        """hexgen2/model.py:73-78 for the hf-reference engine; transformers' DynamicCache
        replaces the tuple cache the reference reads (its layers hold [1, hkv, L, d] keys and
        values), and the cache goes out as {layer: [1, L, 2, hkv, d]} as there."""
        ids = torch.tensor([input_ids], dtype=torch.long, device=self.device)
        result = self.model(ids, use_cache=True)
        cache = {i: torch.stack((l.keys.transpose(1, 2), l.values.transpose(1, 2)), dim=2).contiguous()
                 for i, l in enumerate(result.past_key_values.layers)}
        logits = result.logits[:, -1]
        return logits.argmax(-1), cache, logits

    def _check_live_cache(self, cache, prompt_length):
        """hexgen2/model.py:90-97."""
        if set(cache) != set(range(self.config.num_hidden_layers)):
            raise ValueError("KV cache does not match the configured layer count")
        expected = (1, prompt_length, 2, self.kv_heads, self.head_dim)
        for value in cache.values():
            if tuple(value.shape) != expected or value.dtype != self.dtype:
                raise ValueError("KV cache shape/dtype does not match checkpoint and prompt")

    @torch.inference_mode()
    def decode(self, first_token, cache, prompt_length, max_new_tokens, on_token=None):
        token = first_token.to(self.device).reshape(1)
        generated = [int(token.item())]
        if on_token:
            on_token(generated[-1])
        self._check_live_cache(cache, prompt_length)
        if self.kind == "hf-reference":
            return self._hf_decode(token, cache, max_new_tokens, generated, on_token)
        state = CacheState(prompt_length + max_new_tokens)
        state.sequence_len_offset = prompt_length
        state.key_value_memory_dict = self.unpack_live([dict(cache)], [prompt_length],
                                                       state.max_sequence_len)
        for _ in range(max_new_tokens - 1):
            logits = self.model(token[:, None], inference_params=state, last_token_only=True).logits
            state.sequence_len_offset += 1
            token = ops.argmax(logits)
            generated.append(int(token.item()))
            if on_token:
                on_token(generated[-1])
        return generated

    def _hf_decode(self, token, cache, max_new_tokens, generated, on_token):
        """hexgen2/model.py:98-121 for the hf-reference engine, the live cache handed to
        transformers as a DynamicCache."""
        from transformers import DynamicCache

        past = DynamicCache()
        for i in range(len(cache)):
            kv = cache[i].to(self.device)
            past.update(kv[:, :, 0].transpose(1, 2).contiguous(),
                        kv[:, :, 1].transpose(1, 2).contiguous(), i)
        for _ in range(max_new_tokens - 1):
            result = self.model(token[:, None], past_key_values=past, use_cache=True)
            past, logits = result.past_key_values, result.logits[:, -1]
            token = logits.argmax(-1)
            generated.append(int(token.item()))
            if on_token:
                on_token(generated[-1])
        return generated

    @torch.inference_mode()
    def decode_batch(self, first_tokens: torch.Tensor, caches: dict, lengths: torch.Tensor,
                     steps: int, use_graph: bool = True, capture_first: bool = False):
        """Greedy decode of a ragged batch without host syncs: first_tokens [B] (device int64),
        caches {layer: [B, capacity, 2, hkv, d]} holding lengths[b] live rows per sequence
        (lengths: int32 device [B], advanced in place). Returns tokens [B, steps + 1] on the
        device (column 0 = first_tokens).

        With use_graph, one single-token step is captured in a CUDA graph whose input is a
        static token buffer that the previous replay's argmax wrote and whose length increment
        is part of the graph, so a step is one launch from the host. The graph is kept per
        (batch, cache, lengths, scratch buffers, rotary tables) and replayed by later calls on
        the same buffers; the first call runs one step eagerly (it also sizes every scratch
        buffer) and captures. With capture_first (for callers that already ran a step on these
        buffers, so every scratch buffer is sized), a missing graph is captured at the first
        step instead, so even single-step calls replay."""
        self._native_only("decode_batch")
        B = first_tokens.numel()
        capacity = caches[0].shape[1]
        tokens = torch.empty(steps + 1, B, dtype=torch.long, device=self.device)
        tokens[0] = first_tokens.reshape(B)
        if steps <= 0:
            return tokens.t()

        def graph_key():
            cos = self.model.rope_tables(capacity, self.device, self.dtype)[0]
            return (B, capacity, caches[0].data_ptr(), lengths.data_ptr(), ops.WORKSPACE_GEN,
                    cos.data_ptr())

        graphs = self.__dict__.setdefault("_decode_graphs", {})
        entry = graphs.get(graph_key()) if use_graph else None
        if entry is None:
            state = CacheState(capacity, max_batch_size=B)
            state.key_value_memory_dict = caches
            state.lengths_per_sample = lengths
            cur = torch.empty(B, 1, dtype=torch.long, device=self.device)
        else:
            graph, cur, per_replay = entry
        cur.copy_(tokens[0].view(B, 1))

        def step():
            nxt = self.model.next_tokens(cur, inference_params=state)
            lengths.add_(1)
            cur.view(B).copy_(nxt)

        for s in range(steps):
            if entry is not None:
                graph.replay()
                ops.LAUNCHES += per_replay  # kernels of this library inside one replay
            elif use_graph and (s >= 1 or capture_first):
                graph = torch.cuda.CUDAGraph()
                before = ops.LAUNCHES
                with torch.cuda.graph(graph):
                    step()
                per_replay = ops.LAUNCHES - before  # counted once at capture = first replay
                entry = (graph, cur, per_replay)
                if len(graphs) >= 4:
                    graphs.pop(next(iter(graphs)))
                graphs[graph_key()] = entry
                graph.replay()
            else:
                step()
            tokens[s + 1].copy_(cur.view(B))
        return tokens.t()

    def release_graphs(self):
        """Drops the kept decode graphs (needed before tearing down a process group whose
        collectives they captured)."""
        self.__dict__.pop("_decode_graphs", None)

    @torch.inference_mode()
    def prefill_chunks(self, ids, lengths, cache, first, events=None,
                       max_tokens=PREFILL_TOKENS, max_prompts=PREFILL_PROMPTS):
        """Prefills prompts (flat device ids, prompt b of lengths[b] tokens into batch row b of
        `cache`) in packed passes of at most max_tokens tokens / max_prompts prompts
        (GPTLMHeadModel.prefill_packed), writing each greedy first token into first[b]. With
        events, events[b] is recorded when prompt b's first token is ready."""
        self._native_only("prefill_chunks")
        offs = [0]
        for L in lengths:
            offs.append(offs[-1] + L)
        b0 = 0
        while b0 < len(lengths):
            b1, tok = b0, 0
            while b1 < len(lengths) and b1 - b0 < max_prompts and (
                    b1 == b0 or tok + lengths[b1] <= max_tokens):
                tok += lengths[b1]
                b1 += 1
            self.model.prefill_packed(ids[offs[b0]:offs[b1]], lengths[b0:b1], cache,
                                      list(range(b0, b1)), out=first[b0:b1])
            if events is not None:
                for b in range(b0, b1):
                    events[b].record()
            b0 = b1

    def serve_batch(self, prompts, lengths=None, max_new_tokens=16):
        """Colocated greedy generation for a batch of requests: prompts as a list of token-id
        lists, or a flat (ideally pinned) int64 CPU tensor plus per-request lengths. The
        prompts are prefilled in packed passes straight into their slots of one all-layer
        cache, then the whole ragged batch decodes together. Returns a list of max_new_tokens
        tokens per request."""
        self._native_only("serve_batch")
        if isinstance(prompts, torch.Tensor):
            flat, lens = prompts, list(lengths)
        else:
            lens = [len(p) for p in prompts]
            flat = torch.tensor([t for p in prompts for t in p], dtype=torch.long)
        B = len(lens)
        capacity = max(lens) + max_new_tokens
        ids = flat.to(self.device, non_blocking=True)
        cache = self.model.allocate_inference_cache(B, capacity)
        first = torch.empty(B, dtype=torch.long, device=self.device)
        self.prefill_chunks(ids, lens, cache, first)
        lengths_dev = torch.tensor(lens, dtype=torch.int32).to(self.device, non_blocking=True)
        toks = self.decode_batch(first, cache, lengths_dev, max_new_tokens - 1)
        return toks.cpu().tolist()

    def synchronize(self):
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)


class ContinuousBatcher:
    """Continuous batching on one engine: a fixed pool of `slots` sequences in one all-layer
    cache [layers, slots, capacity, 2, hkv, d]. Every step decodes all slots with one replay
    of the kept decode graph (ragged per-slot lengths); a finished request frees its slot at
    once, and waiting requests are prefilled straight into free slots between steps. Idle
    slots sit at length 0 (their step attends to one key and is discarded).

    The reference batches by padding every cache to the longest one and decoding the padded
    batch until all requests end (hexgen/llama/kv_cache_batch.py:4-29,
    inference_phases.py:141-212); here requests join and leave per step, and each request's
    tokens equal its batch-1 greedy decode.
    """

    def __init__(self, engine: Engine, slots: int, capacity: int):
        engine._native_only("ContinuousBatcher")
        self.eng, self.slots, self.capacity = engine, slots, capacity
        dev = engine.device
        self.cache = engine.model.allocate_inference_cache(slots, capacity)
        self.lengths = torch.zeros(slots, dtype=torch.int32, device=dev)
        self.tokens = torch.zeros(slots, dtype=torch.long, device=dev)
        self.req = [None] * slots        # request id per slot
        self.left = [0] * slots          # tokens still to generate per slot
        self.out: dict = {}              # request id -> generated tokens
        # Capture the decode graph once on the idle pool; later steps only replay it.
        self.eng.decode_batch(self.tokens, self.cache, self.lengths, 2)
        self.lengths.zero_()

    def free_slots(self) -> list[int]:
        return [i for i, r in enumerate(self.req) if r is None]

    def active(self) -> int:
        return sum(r is not None for r in self.req)

    @torch.inference_mode()
    def admit(self, req_id, prompt: list[int], max_new_tokens: int) -> int:
        """Prefills `prompt` into a free slot; returns the first generated token (greedy)."""
        free = self.free_slots()
        if not free:
            raise ValueError("no free slot")
        L = len(prompt)
        if L + max_new_tokens > self.capacity:
            raise ValueError(f"request needs {L + max_new_tokens} positions, capacity {self.capacity}")
        slot = free[0]
        ids = torch.tensor([prompt], dtype=torch.long, device=self.eng.device)
        st = CacheState(self.capacity, max_batch_size=self.slots, batch_size_offset=slot,
                        key_value_memory_dict=self.cache)
        logits = self.eng.model(ids, inference_params=st, last_token_only=True).logits
        ops.argmax(logits, out=self.tokens[slot:slot + 1])
        self.lengths[slot:slot + 1].fill_(L)
        first = int(self.tokens[slot].item())
        self.req[slot], self.left[slot] = req_id, max_new_tokens - 1
        self.out[req_id] = [first]
        if self.left[slot] == 0:
            self._retire(slot)
        return first

    @torch.inference_mode()
    def admit_packed(self, req_id, src, src_offset: int, length: int, first_token: int,
                     max_new_tokens: int) -> int:
        """Admits a request prefilled elsewhere into a free slot: its live rows of every layer,
        packed as Engine.pack_live and the prefill rank's gather-pack write them ([layers][L]
        rows of [2, hkv, d] at byte offset src_offset of `src`, a CUDA tensor or a device
        address on this GPU), are scattered into the slot with one kernel, and decoding
        continues from first_token. Returns the slot."""
        free = self.free_slots()
        if not free:
            raise ValueError("no free slot")
        if length + max_new_tokens > self.capacity:
            raise ValueError(f"request needs {length + max_new_tokens} positions, capacity {self.capacity}")
        slot = free[0]
        dev = self.eng.device
        big0 = self.cache[0]
        elem = big0.element_size()
        n = self.eng.num_layers
        layer_stride = self.cache[1].data_ptr() - big0.data_ptr() if n > 1 else 0
        dst = torch.tensor([big0.data_ptr() + slot * big0.stride(0) * elem], dtype=torch.int64,
                           device=dev)
        ops.kv_unpack(src, torch.tensor([src_offset], dtype=torch.int64, device=dev),
                      torch.tensor([length], dtype=torch.int64, device=dev), dst, n, layer_stride,
                      big0.stride(1) * elem, self.eng.row_bytes, length)
        self.tokens[slot:slot + 1].fill_(first_token)
        self.lengths[slot:slot + 1].fill_(length)
        self.req[slot], self.left[slot] = req_id, max_new_tokens - 1
        self.out[req_id] = [first_token]
        if self.left[slot] == 0:
            self._retire(slot)
        return slot

    def _retire(self, slot: int):
        self.req[slot] = None
        self.lengths[slot:slot + 1].zero_()

    @torch.inference_mode()
    def step(self) -> list:
        """One decode step for every slot; returns the ids of requests that finished."""
        toks = self.eng.decode_batch(self.tokens, self.cache, self.lengths, 1, capture_first=True)
        new = toks[:, 1].contiguous()
        self.tokens.copy_(new)
        host = new.tolist()
        done = []
        for slot, rid in enumerate(self.req):
            if rid is None:
                continue
            self.out[rid].append(host[slot])
            self.left[slot] -= 1
            if self.left[slot] == 0:
                self._retire(slot)
                done.append(rid)
        return done


def serve_arrivals(batcher: ContinuousBatcher, requests: list, clock=None) -> dict:
    """Serves requests [(req_id, prompt, max_new_tokens, arrival_s)] as they arrive (wall clock
    from the first call), admitting into free slots between decode steps. Returns per request
    {"tokens", "ttft_s", "done_s"} (times relative to the start)."""
    import time
    clock = clock or time.perf_counter
    t0 = clock()
    pending = sorted(requests, key=lambda r: r[3])
    stats, arrival = {}, {r[0]: r[3] for r in requests}
    i = 0
    while i < len(pending) or batcher.active():
        now = clock() - t0
        while i < len(pending) and pending[i][3] <= now and batcher.free_slots():
            rid, prompt, max_new, _ = pending[i]
            batcher.admit(rid, prompt, max_new)
            stats[rid] = {"ttft_s": clock() - t0 - arrival[rid]}
            if batcher.req.count(rid) == 0:  # finished at its first token
                stats[rid]["done_s"] = clock() - t0
            i += 1
        if batcher.active():
            for rid in batcher.step():
                stats[rid]["done_s"] = clock() - t0
        elif i < len(pending):
            wait = pending[i][3] - (clock() - t0)
            if wait > 0:
                time.sleep(min(wait, 0.01))
    for rid in stats:
        stats[rid]["tokens"] = batcher.out[rid]
    return stats
