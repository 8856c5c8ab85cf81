"""End-to-end parity on the GPU: the Engine / GPTLMHeadModel drop-in against the reference's
golden vectors (seed-0 fixture) and against the CPU oracle on seeded random-weight models of
the BASELINE architectures (reduced layer counts so the oracle finishes in seconds).

Parity bars: logits within 1e-4 (f32) / 2e-2 (bf16) of the reference,
in the reference's own acceptance form |a - b| <= atol + rtol * |b| with atol = rtol
(hexgen2/validate.py:43 uses 0.03 for both). On the fixture (and in f32) that bound is asserted
for every logit. At full architecture width it cannot hold for every logit in bf16, for any
implementation that does not reproduce cuBLAS's and FlashAttention's exact f32 summation order:
two restatements of the reference itself (its CPU torch attention vs FlashAttention numerics)
already differ by up to 0.043 (TinyLlama width) and 0.086-0.107 (7B width) after two layers,
with only ~70% of 7B-width logits within 2e-2 of each other. There the asserted bar is: the
max error is within max(2e-2, the reference's own spread), the fraction of logits within 2e-2
(atol = rtol form) is at least the reference's own (capped at 99%), and greedy tokens are
identical except at a near-tie of the reference's own logits (top-2 margin inside the
tolerance), which is reported.
"""
import pytest
import torch

from oracle.llama_ref import LlamaShape, OracleModel, random_native_state
from tests.conftest import from_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def hx():
    import hexgen2_b200
    return hexgen2_b200


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
def test_engine_prefill_matches_reference_golden(hx, golden, fixture_dir, dtype):
    """Prefill logits against the reference's golden bits and the returned cache shapes.
    Decode logits and greedy tokens are checked step by step in test_parity_gpu.py."""
    eng = hx.Engine(fixture_dir, device="cuda", dtype=dtype)
    tol = 1e-4 if dtype == "float32" else 2e-2
    for row in golden["engine"][dtype]:
        first, cache, logits = eng.prefill(row["prompt"], row["max_new"])
        expected = from_bits(row["prefill_logits"], getattr(torch, dtype)).float()
        torch.testing.assert_close(logits[0].float().cpu(), expected, rtol=0, atol=tol)
        for k, meta in row["kv"].items():
            assert list(cache[int(k)].shape) == meta["shape"]
        if dtype == "float32":
            assert int(first) == row["first_token"]


def test_prefill_cache_matches_reference_in_f32(hx, golden, fixture_dir):
    """Layer-0 K/V rows of the reference's f32 prefill (golden values of the short prompts),
    within 1e-5."""
    eng = hx.Engine(fixture_dir, device="cuda", dtype="float32")
    for row in golden["engine"]["float32"]:
        _, cache, _ = eng.prefill(row["prompt"], row["max_new"])
        if row["kv_layer0_values"] is not None:
            expected = from_bits(row["kv_layer0_values"], torch.float32)
            torch.testing.assert_close(cache[0].cpu().flatten(), expected, rtol=0, atol=1e-5)


def _oracle_and_engine(hx, shape_kwargs, layers, dtype, seed):
    shape = LlamaShape(**shape_kwargs)
    shape.num_layers = layers
    state = random_native_state(shape, seed=seed, dtype=dtype)
    oracle = OracleModel(shape, state, dtype, attention="flash")
    cfg = dict(vocab_size=shape.vocab_size, hidden_size=shape.hidden_size,
               intermediate_size=shape.intermediate_size, num_hidden_layers=layers,
               num_attention_heads=shape.num_heads, num_key_value_heads=shape.num_kv_heads,
               rms_norm_eps=shape.rms_norm_eps, rope_theta=shape.rope_theta,
               max_position_embeddings=8192)
    from hexgen2_b200.checkpoint import llama_config_to_gpt2_config
    from transformers import LlamaConfig
    gcfg = llama_config_to_gpt2_config(LlamaConfig(**cfg))
    model = hx.GPTLMHeadModel(gcfg, device="cuda", dtype=dtype).eval()
    model.load_state_dict({k: v.cuda() for k, v in state.items()}, strict=True)
    eng = hx.Engine.__new__(hx.Engine)
    eng.device, eng.dtype, eng.model, eng.kind = torch.device("cuda"), dtype, model, "native"
    eng.config = LlamaConfig(**cfg)
    eng._post_init()
    return oracle, eng


TINYLLAMA = dict(vocab_size=32000, hidden_size=2048, intermediate_size=5632, num_layers=22,
                 num_heads=32, num_kv_heads=4, rms_norm_eps=1e-5, rope_theta=10000.0)
LLAMA7B = dict(vocab_size=32000, hidden_size=4096, intermediate_size=11008, num_layers=32,
               num_heads=32, num_kv_heads=32, rms_norm_eps=1e-5, rope_theta=10000.0)
LLAMA70B_TP4_SHARD = dict(vocab_size=32000, hidden_size=8192, intermediate_size=28672, num_layers=80,
                          num_heads=64, num_kv_heads=8, rms_norm_eps=1e-5, rope_theta=10000.0)


def _teacher_forced_check(oracle, eng, prompt, steps, tol, noise_oracle=None):
    """Runs the engine's greedy decode, then replays the engine's token sequence through the
    oracle: logits must agree at every step (atol = rtol = tol), and any token divergence must
    sit on a near-tie of the oracle's own logits. With noise_oracle (the reference's other
    attention numerics) the CUDA path's max error must not exceed the reference's own spread.
    Returns the list of near-tie steps."""
    first, cache, logits = eng.prefill(prompt, steps)
    tokens = eng.decode(first, cache, len(prompt), steps)
    o_first, o_cache, o_logits = oracle.prefill(prompt, steps)
    got, ref = logits[0].float().cpu(), o_logits[0].float()
    if noise_oracle is None:
        torch.testing.assert_close(got, ref, rtol=tol, atol=tol)
    else:
        _, _, n_logits = noise_oracle.prefill(prompt, steps)
        floor = (n_logits[0].float() - ref).abs().max().item()
        diff = (got - ref).abs()
        err = diff.max().item()
        within = (diff <= tol + tol * ref.abs()).float().mean().item()
        n_diff = (n_logits[0].float() - ref).abs()
        within_floor = (n_diff <= tol + tol * ref.abs()).float().mean().item()
        print(f"max |logit err| {err:.4f} (reference's own spread {floor:.4f}); "
              f"{within:.4%} of logits within {tol} (reference vs itself: {within_floor:.4%})")
        assert err <= max(floor, tol), (err, floor)
        assert within >= min(within_floor, 0.99), (within, within_floor)
    ties = []
    ids = torch.tensor([prompt + tokens[:-1]])
    full = oracle.forward(ids, None, last_token_only=False)[0].float()
    for s, tok in enumerate(tokens):
        row = full[len(prompt) - 1 + s]
        top2 = row.topk(2)
        if int(top2.indices[0]) != tok:
            margin = float(top2.values[0] - row[tok])
            assert margin <= tol + tol * float(top2.values[0].abs()), (s, tok, int(top2.indices[0]), margin)
            ties.append((s, margin))
    return ties


@pytest.mark.parametrize("arch,layers", [("tinyllama", 2), ("llama7b", 2)])
def test_bf16_parity_against_oracle(hx, arch, layers):
    shape = TINYLLAMA if arch == "tinyllama" else LLAMA7B
    oracle, eng = _oracle_and_engine(hx, shape, layers, torch.bfloat16, seed=1)
    noise = OracleModel(oracle.shape, {k: v for k, v in oracle.w.items()}, torch.bfloat16,
                        attention="torch")
    g = torch.Generator().manual_seed(5)
    for L in (8, 77, 300):
        prompt = torch.randint(0, 32000, (L,), generator=g).tolist()
        ties = _teacher_forced_check(oracle, eng, prompt, 6, 2e-2, noise_oracle=noise)
        print(arch, L, "near-ties:", ties)


def test_f32_parity_against_oracle(hx):
    shape = dict(TINYLLAMA, vocab_size=4096, hidden_size=512, intermediate_size=1024,
                 num_heads=8, num_kv_heads=2)
    oracle, eng = _oracle_and_engine(hx, shape, 2, torch.float32, seed=2)
    prompt = list(range(3, 40))
    first, cache, logits = eng.prefill(prompt, 8)
    o_first, o_cache, o_logits = oracle.prefill(prompt, 8)
    torch.testing.assert_close(logits.cpu(), o_logits, rtol=0, atol=1e-4)
    for i in cache:
        torch.testing.assert_close(cache[i].cpu(), o_cache[i], rtol=0, atol=1e-5)
    assert eng.decode(first, cache, len(prompt), 8) == oracle.decode(o_first, o_cache, len(prompt), 8)


def test_gqa_70b_shard_shape_one_layer(hx):
    """One layer of the Llama-2-70B TP4 shard geometry (16 q heads / 2 kv heads per rank)."""
    shape = dict(LLAMA70B_TP4_SHARD, vocab_size=8192, hidden_size=2048, intermediate_size=7168,
                 num_heads=16, num_kv_heads=2)
    oracle, eng = _oracle_and_engine(hx, shape, 1, torch.bfloat16, seed=3)
    _teacher_forced_check(oracle, eng, list(range(100, 160)), 4, 2e-2)


def test_disaggregated_equals_colocated(hx, fixture_dir):
    """Prefill on one engine, transfer the packed live cache, decode on another == colocated."""
    a = hx.Engine(fixture_dir, device="cuda", dtype="bfloat16")
    b = hx.Engine(fixture_dir, device="cuda", dtype="bfloat16")
    prompt = [1, 8, 9, 10, 44, 2, 7]
    first, cache, _ = a.prefill(prompt, 12)
    moved = {k: v.clone() for k, v in cache.items()}
    del cache
    seen = []  # on_token sees every generated token in order, the first one included
    t1 = b.decode(first, moved, len(prompt), 12, on_token=seen.append)
    assert seen == t1
    f2, c2, _ = a.prefill(prompt, 12)
    t2 = a.decode(f2, c2, len(prompt), 12)
    assert t1 == t2


def test_decode_batch_ragged_matches_single(hx):
    oracle, eng = _oracle_and_engine(hx, dict(TINYLLAMA, vocab_size=4096), 2, torch.bfloat16, seed=4)
    prompts = [list(range(5, 5 + L)) for L in (9, 40, 3, 64)]
    steps = 10
    singles, firsts, caches, lens = [], [], [], []
    for p in prompts:
        f, c, _ = eng.prefill(p, steps + 1)
        singles.append(eng.decode(f, {k: v.clone() for k, v in c.items()}, len(p), steps + 1))
        firsts.append(f)
        caches.append(c)
        lens.append(len(p))
    full = eng.unpack_live(caches, lens, max(lens) + steps + 1)
    lengths = torch.tensor(lens, dtype=torch.int32, device="cuda")
    toks = eng.decode_batch(torch.cat(firsts), full, lengths, steps).cpu().tolist()
    for s, t in zip(singles, toks):
        assert s == t
    assert lengths.cpu().tolist() == [L + steps for L in lens]


def test_tp_rejects_bad_sizes(hx):
    from hexgen2_b200.checkpoint import shard_state_dict_tp
    with pytest.raises(AssertionError):
        class C:
            n_head, n_head_kv, n_embd, vocab_size, n_layer = 6, 6, 48, 10, 1
        shard_state_dict_tp({}, C, 4, 0)


def test_decode_graph_is_kept_and_replayed(hx):
    """A second decode_batch on the same buffers replays the kept CUDA graph (no recapture)
    and produces the same tokens as the first call and as an eager run."""
    oracle, eng = _oracle_and_engine(hx, dict(TINYLLAMA, vocab_size=4096), 2, torch.bfloat16, seed=6)
    prompts = [list(range(7, 7 + L)) for L in (33, 5, 90)]
    firsts, caches, lens = [], [], []
    for p in prompts:
        f, c, _ = eng.prefill(p, 16)
        firsts.append(f)
        caches.append(c)
        lens.append(len(p))
    steps = 12
    full = eng.unpack_live(caches, lens, max(lens) + steps + 1)
    first = torch.cat(firsts)
    lengths = torch.tensor(lens, dtype=torch.int32, device="cuda")
    runs = []
    for use_graph in (True, True, False):
        lengths.copy_(torch.tensor(lens, dtype=torch.int32))
        runs.append(eng.decode_batch(first, full, lengths, steps, use_graph=use_graph).cpu().tolist())
        if use_graph:
            assert len(eng._decode_graphs) == 1
    assert runs[0] == runs[1] == runs[2]
    eng.release_graphs()
    assert not getattr(eng, "_decode_graphs", None)


def test_continuous_batching_matches_batch1_greedy(hx):
    """Six requests through three slots (requests join as slots free up, one finishes at its
    first token): every request's tokens equal its own batch-1 prefill + greedy decode."""
    oracle, eng = _oracle_and_engine(hx, dict(TINYLLAMA, vocab_size=4096), 2, torch.bfloat16, seed=7)
    g = torch.Generator().manual_seed(9)
    reqs = [(i, torch.randint(0, 4096, (L,), generator=g).tolist(), n)
            for i, (L, n) in enumerate([(5, 7), (40, 3), (17, 12), (3, 1), (64, 9), (9, 6)])]
    expected = {}
    for rid, prompt, n in reqs:
        f, c, _ = eng.prefill(prompt, n)
        expected[rid] = eng.decode(f, c, len(prompt), n)
    batcher = hx.ContinuousBatcher(eng, slots=3, capacity=80)
    stats = hx.serve_arrivals(batcher, [(rid, p, n, 0.0) for rid, p, n in reqs])
    for rid, p, n in reqs:
        assert stats[rid]["tokens"] == expected[rid], rid
        assert stats[rid]["ttft_s"] >= 0 and stats[rid]["done_s"] >= stats[rid]["ttft_s"]
    assert batcher.active() == 0 and len(batcher.free_slots()) == 3
    assert len(eng._decode_graphs) == 1  # one kept graph served every step
