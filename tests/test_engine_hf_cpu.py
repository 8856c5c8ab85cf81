"""The reference's `hf-reference` validation engine through this package's Engine, on the CPU
(hexgen2/model.py:32-37, :73-78, :98-121): chosen explicitly, it gives the golden fixture's
prefill logits and greedy tokens as the reference's Engine does, hands the cache out in the
reference's live layout, and the native-only entry points refuse it."""
import pytest
import torch

import hexgen2_b200 as hx
from hexgen2_b200.engine import ContinuousBatcher
from tests.conftest import from_bits


@pytest.fixture(scope="module")
def hf_engine(fixture_dir):
    return hx.Engine(fixture_dir, engine="hf-reference", device="cpu", dtype="float32")


def test_hf_reference_engine_matches_goldens_f32(hf_engine, golden):
    cfg = golden["fixture_config"]
    kv, d = cfg["num_key_value_heads"], cfg["hidden_size"] // cfg["num_attention_heads"]
    for row in golden["engine"]["float32"]:
        L = len(row["prompt"])
        first, cache, logits = hf_engine.prefill(row["prompt"], row["max_new"])
        want = from_bits(row["prefill_logits"], torch.float32)
        # The reference's own HF-eager / native difference on these prompts is <= 4.2e-7.
        assert (logits[0].float() - want).abs().max().item() <= 1e-5, row["name"]
        assert int(first) == row["first_token"], row["name"]
        assert set(cache) == set(range(cfg["num_hidden_layers"]))
        assert all(tuple(c.shape) == (1, L, 2, kv, d) for c in cache.values())
        tokens = hf_engine.decode(first, cache, L, row["max_new"])
        assert tokens == row["tokens"] == row["hf_eager_tokens"], row["name"]


def test_hf_reference_engine_checks_the_cache(hf_engine, golden):
    row = golden["engine"]["float32"][1]
    first, cache, _ = hf_engine.prefill(row["prompt"], row["max_new"])
    with pytest.raises(ValueError):
        hf_engine.decode(first, cache, len(row["prompt"]) + 1, row["max_new"])
    with pytest.raises(ValueError):
        hf_engine.decode(first, {0: cache[0]}, len(row["prompt"]), row["max_new"])


def test_native_only_entry_points_refuse_hf_reference(hf_engine, fixture_dir):
    with pytest.raises(ValueError):
        hf_engine.serve_batch([[1, 2, 3]], max_new_tokens=2)
    with pytest.raises(ValueError):
        ContinuousBatcher(hf_engine, 2, 16)
    with pytest.raises(ValueError):
        hx.Engine(fixture_dir, engine="bogus", device="cpu", dtype="float32")
