"""Host-side model plumbing on the CPU: HF -> native remap (against the oracle's restatement
and the reference's goldens), TP sharding semantics on real 2-rank Gloo groups, the SwiGLU
weight interleave and the reference-compatible state dict."""
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hexgen2_b200.checkpoint import (config_from_dict, remap_state_dict_hf_llama,
                                     shard_state_dict_tp)
from hexgen2_b200.gpt import GPTLMHeadModel, deinterleave_gated, interleave_gated
from oracle.llama_ref import LlamaShape, random_native_state, remap_hf_to_native

SMALL = dict(vocab_size=64, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
             num_attention_heads=4, num_key_value_heads=2, rms_norm_eps=1e-5)


def test_remap_matches_oracle(fixture_dir):
    from safetensors.torch import load_file
    from hexgen2_b200.checkpoint import llama_config_to_gpt2_config
    from transformers import LlamaConfig
    raw = {}
    for s in sorted(Path(fixture_dir).glob("*.safetensors")):
        raw.update(load_file(str(s)))
    cfg = llama_config_to_gpt2_config(LlamaConfig.from_pretrained(fixture_dir))
    ours = remap_state_dict_hf_llama(dict(raw), cfg)
    theirs = remap_hf_to_native(dict(raw), LlamaShape.from_hf(LlamaConfig.from_pretrained(fixture_dir)))
    assert set(ours) == set(theirs)
    for k in ours:
        assert torch.equal(ours[k], theirs[k]), k


def test_interleave_roundtrip():
    w = torch.arange(64 * 3).reshape(64, 3).float()
    iw = interleave_gated(w)
    assert torch.equal(iw[:16], w[:16]) and torch.equal(iw[16:32], w[32:48])
    assert torch.equal(deinterleave_gated(iw), w)


def test_model_state_dict_is_reference_layout():
    cfg = config_from_dict(SMALL)
    model = GPTLMHeadModel(cfg, device="cpu", dtype=torch.float32)
    shape = LlamaShape.from_hf(SMALL)
    state = random_native_state(shape, seed=0)
    model.load_state_dict(state, strict=True)
    back = model.state_dict()
    assert set(back) == set(state)
    for k in state:
        assert torch.equal(back[k], state[k]), k
    # Internally fc1 is interleaved for the SwiGLU epilogue.
    w = model.transformer.layers[0].mlp.fc1.weight
    assert torch.equal(w, interleave_gated(state["transformer.layers.0.mlp.fc1.weight"]))


def _tp_worker(rank, rendezvous):
    dist.init_process_group("gloo", rank=rank, world_size=2, init_method=Path(rendezvous).as_uri(),
                            timeout=timedelta(seconds=30))
    try:
        cfg = config_from_dict(dict(SMALL, num_key_value_heads=2))
        full = random_native_state(LlamaShape.from_hf(SMALL), seed=1)
        shard = shard_state_dict_tp(dict(full), cfg, 2, rank)
        x = torch.randn(3, 64, generator=torch.Generator().manual_seed(9))
        # Column-parallel Wqkv: each rank holds its heads' q, k, v rows.
        q_full = x @ full["transformer.layers.0.mixer.Wqkv.weight"].T
        q_loc = x @ shard["transformer.layers.0.mixer.Wqkv.weight"].T
        d, hq, hk = 16, 4, 2
        parts = [torch.empty_like(q_loc) for _ in range(2)]
        dist.all_gather(parts, q_loc)
        qs = [p[:, : (hq // 2) * d] for p in parts]
        ks = [p[:, (hq // 2) * d:(hq // 2 + hk // 2) * d] for p in parts]
        assert torch.allclose(torch.cat(qs, 1), q_full[:, : hq * d], atol=1e-6)
        assert torch.allclose(torch.cat(ks, 1), q_full[:, hq * d:(hq + hk) * d], atol=1e-6)
        # Row-parallel out_proj + all-reduce == full out_proj.
        c = torch.randn(3, 64, generator=torch.Generator().manual_seed(10))
        w_full = full["transformer.layers.0.mixer.out_proj.weight"]
        w_loc = shard["transformer.layers.0.mixer.out_proj.weight"]
        part = c[:, rank * 32:(rank + 1) * 32] @ w_loc.T
        dist.all_reduce(part)
        assert torch.allclose(part, c @ w_full.T, atol=1e-5)
        # fc1 halves: rank holds matching up/gate rows.
        f_full = full["transformer.layers.0.mlp.fc1.weight"]
        f_loc = shard["transformer.layers.0.mlp.fc1.weight"]
        assert torch.equal(f_loc[:64], f_full[rank * 64:(rank + 1) * 64])
        assert torch.equal(f_loc[64:], f_full[128 + rank * 64:128 + (rank + 1) * 64])
        # Vocab-parallel embedding rows.
        e_loc = shard["transformer.embeddings.word_embeddings.weight"]
        assert torch.equal(e_loc, full["transformer.embeddings.word_embeddings.weight"][rank * 32:(rank + 1) * 32])
        # The TP model builds on each rank and accepts its shard strictly.
        with torch.device("meta"):
            m = GPTLMHeadModel(cfg, process_group=dist.group.WORLD, dtype=torch.float32)
        m.load_state_dict(shard, strict=True, assign=True)
        assert m.transformer.layers[0].mixer.Wqkv.weight.shape == (64 // 2 + 2 * 16, 64)
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_sharding_on_two_gloo_ranks(tmp_path):
    mp.spawn(_tp_worker, args=(str(tmp_path / "rv"),), nprocs=2, join=True)


def _hf_state(cfg: dict, seed: int, with_lm_head: bool = True) -> dict:
    """A small HF-named Llama state dict (seeded N(0, 0.02))."""
    g = torch.Generator().manual_seed(seed)
    h, I, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    d = h // cfg["num_attention_heads"]
    hk = cfg["num_key_value_heads"]

    def rnd(*s):
        return torch.randn(*s, generator=g) * 0.02

    sd = {"model.embed_tokens.weight": rnd(V, h), "model.norm.weight": torch.ones(h)}
    if with_lm_head:
        sd["lm_head.weight"] = rnd(V, h)
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}."
        sd.update({p + "input_layernorm.weight": torch.ones(h),
                   p + "post_attention_layernorm.weight": torch.ones(h),
                   p + "self_attn.q_proj.weight": rnd(h, h),
                   p + "self_attn.k_proj.weight": rnd(hk * d, h),
                   p + "self_attn.v_proj.weight": rnd(hk * d, h),
                   p + "self_attn.o_proj.weight": rnd(h, h),
                   p + "mlp.gate_proj.weight": rnd(I, h), p + "mlp.up_proj.weight": rnd(I, h),
                   p + "mlp.down_proj.weight": rnd(h, I)})
    return sd


ODD_VOCAB = dict(SMALL, vocab_size=61)


@pytest.mark.parametrize("tied", [False, True])
def test_remap_pads_vocab_and_ties_like_reference(tied):
    """remap_state_dict.py:28-51: embedding and LM head zero-padded to pad_vocab_size_multiple
    rows; tie_word_embeddings makes the LM head the (padded) embedding."""
    cfg = config_from_dict(ODD_VOCAB)
    cfg.pad_vocab_size_multiple = 8
    cfg.tie_word_embeddings = tied
    sd = _hf_state(ODD_VOCAB, seed=3, with_lm_head=not tied)
    out = remap_state_dict_hf_llama(dict(sd), cfg)
    emb, head = out["transformer.embeddings.word_embeddings.weight"], out["lm_head.weight"]
    assert emb.shape[0] == 64 and head.shape[0] == 64
    assert torch.equal(emb[:61], sd["model.embed_tokens.weight"]) and not emb[61:].any()
    if tied:
        assert head is emb
    else:
        assert torch.equal(head[:61], sd["lm_head.weight"]) and not head[61:].any()
    # The padded state dict loads strictly into the model (which pads its vocab the same way).
    model = GPTLMHeadModel(cfg, device="cpu", dtype=torch.float32)
    model.load_state_dict(out, strict=True)


def test_remap_untied_without_lm_head_raises():
    """With tie_word_embeddings False a checkpoint without lm_head.weight is an error, as in the
    reference (it pops the key unconditionally)."""
    cfg = config_from_dict(SMALL)
    with pytest.raises(KeyError):
        remap_state_dict_hf_llama(_hf_state(SMALL, seed=4, with_lm_head=False), cfg)


REF_REMAP = Path("/root/reference/hexgen/llama/load_model_parameters_utils/remap_state_dict.py")


@pytest.mark.skipif(not REF_REMAP.exists(), reason="reference sources not mounted")
@pytest.mark.parametrize("tied,multiple", [(False, 1), (False, 8), (True, 8)])
def test_remap_equals_reference_remap(tied, multiple):
    """The reference's own remap (imported from its source file) and this one produce the same
    tensors for padded and tied configurations."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("_ref_remap", REF_REMAP)
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    cfg = config_from_dict(ODD_VOCAB)
    cfg.pad_vocab_size_multiple = multiple
    cfg.tie_word_embeddings = tied
    sd = _hf_state(ODD_VOCAB, seed=5, with_lm_head=not tied)
    ours = remap_state_dict_hf_llama(dict(sd), cfg)
    theirs = ref.remap_state_dict_hf_llama(dict(sd), cfg)
    assert set(ours) == set(theirs)
    for k in theirs:
        assert torch.equal(ours[k], theirs[k]), k


@pytest.mark.parametrize("world", [2, 4])
def test_random_init_gives_every_tp_layout_the_same_model(world):
    """random_native_state with tp_world > 1 slices each seeded full tensor to the rank's shard,
    so the TP ranks of a random-init model together hold exactly the TP-1 model (what the
    multi-GPU serving runs rely on when they compare TP decode groups with a colocated run)."""
    from hexgen2_b200.checkpoint import config_from_dict, random_native_state, shard_state_dict_tp
    cfg = config_from_dict(dict(SMALL, num_key_value_heads=4, vocab_size=64))
    full = random_native_state(cfg, seed=3, dtype=torch.float32, device="cpu")
    for rank in range(world):
        part = random_native_state(cfg, seed=3, dtype=torch.float32, device="cpu",
                                   tp_world=world, tp_rank=rank)
        want = shard_state_dict_tp(full, cfg, world, rank)
        assert set(part) == set(want)
        for k in want:
            assert torch.equal(part[k], want[k]), (rank, k)
