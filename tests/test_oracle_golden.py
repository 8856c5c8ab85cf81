"""Pins the CPU oracle to golden vectors produced by the HexGen-2 reference itself.

The oracle (oracle/llama_ref.py) must reproduce the reference's Engine.prefill/decode on the
seed-0 fixture bit for bit in f32, bf16 and f16: greedy tokens, prefill logits and KV bytes.
"""
import hashlib

import pytest
import torch

from oracle.llama_ref import OracleModel, load_hf_checkpoint, rms_norm
from tests.conftest import from_bits

DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def sha(t):
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


@pytest.mark.parametrize("dtype", list(DTYPES))
def test_oracle_matches_reference_engine(golden, fixture_dir, dtype):
    torch.set_num_threads(1)
    shape, state = load_hf_checkpoint(fixture_dir)
    model = OracleModel(shape, state, DTYPES[dtype], attention="torch")
    for row in golden["engine"][dtype]:
        first, cache, logits = model.prefill(row["prompt"], row["max_new"])
        assert int(first) == row["first_token"], row["name"]
        expected = from_bits(row["prefill_logits"], DTYPES[dtype])
        torch.testing.assert_close(logits[0], expected, rtol=0, atol=0, msg=row["name"])
        for k, meta in row["kv"].items():
            assert list(cache[int(k)].shape) == meta["shape"]
            assert sha(cache[int(k)]) == meta["sha256"], (row["name"], k)
        tokens = model.decode(first, cache, len(row["prompt"]), row["max_new"])
        assert tokens == row["tokens"], row["name"]


def test_oracle_flash_mode_agrees_in_f32(golden, fixture_dir):
    """The FlashAttention-numerics mode equals the reference to f32 rounding."""
    shape, state = load_hf_checkpoint(fixture_dir)
    model = OracleModel(shape, state, torch.float32, attention="flash")
    for row in golden["engine"]["float32"]:
        first, cache, logits = model.prefill(row["prompt"], row["max_new"])
        expected = from_bits(row["prefill_logits"], torch.float32)
        torch.testing.assert_close(logits[0], expected, rtol=0, atol=1e-5)
        assert model.decode(first, cache, len(row["prompt"]), row["max_new"]) == row["tokens"]


def test_oracle_rmsnorm_matches_reference_kat(golden):
    for row in golden["rmsnorm"]:
        dtype = {"torch.float32": torch.float32, "torch.float16": torch.float16,
                 "torch.bfloat16": torch.bfloat16}[row["dtype"]]
        x = from_bits(row["input"], dtype).reshape(1, 7, 128)
        w = from_bits(row["weight"], dtype)
        out = rms_norm(x, w, row["eps"])
        torch.testing.assert_close(out.flatten(), from_bits(row["output"], dtype), rtol=0, atol=0)


def test_kv_packet_bytes_closed_form(golden):
    """kv_packet_bytes = 8 (first token) + layers * L * 2 * hkv * d * elem (hexgen2/run.py:147)."""
    for p in golden["transport"]:
        elem = {"float16": 2, "bfloat16": 2, "float32": 4}[p["dtype"]]
        assert p["payload_bytes"] == 8 + 2 * 4 * 2 * 2 * 32 * elem


def test_ragged_batch_decode_equals_per_request_decode(fixture_dir):
    """oracle.RaggedBatch (the CPU baseline's batched decode) gives every request the logits of
    its own batch-1 decode (model.py:85-121 flow), in f32."""
    from oracle.llama_ref import CacheState, RaggedBatch
    shape, state = load_hf_checkpoint(fixture_dir)
    model = OracleModel(shape, state, torch.float32, attention="torch")
    prompts = [[5, 9, 2], list(range(1, 20)), [7]]
    steps = 4
    caches, lens, firsts, singles = [], [], [], []
    for p in prompts:
        st = CacheState(len(p) + steps + 1)
        logits = model.forward(torch.tensor([p]), st, last_token_only=True)
        caches.append(st.key_value_memory_dict)
        lens.append(len(p))
        firsts.append(int(logits.argmax(-1)))
        f, c, _ = model.prefill(p, steps + 1)
        singles.append(model.decode(f, c, len(p), steps + 1, return_logits=True)[1])
    batch = RaggedBatch(model, caches, lens)
    tok = torch.tensor(firsts)
    for s in range(steps):
        logits = batch.step(tok)
        for b in range(len(prompts)):
            torch.testing.assert_close(logits[b], singles[b][s][0], rtol=0, atol=1e-5)
        tok = logits.argmax(-1)
