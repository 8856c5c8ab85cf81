"""Seeded tiny Llama checkpoint for correctness tests (mirrors hexgen2/fixture.py:10-17).

The shapes are the ones the reference fixture writes to its config.json: vocab 128, hidden 128,
intermediate 256, 2 layers, 4 attention heads, 2 KV heads (head_dim 32), 128 positions. The
weights are Hugging Face LlamaForCausalLM default initialisation under torch.manual_seed(seed),
saved as safetensors, exactly like the reference fixture, so the same seed gives the same
checkpoint on any machine with the same torch/transformers.
"""
from __future__ import annotations

import argparse
import hashlib
import json
from pathlib import Path

import torch

FIXTURE_CONFIG = dict(vocab_size=128, hidden_size=128, intermediate_size=256,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      max_position_embeddings=128, bos_token_id=1, eos_token_id=2,
                      pad_token_id=0)


def create(folder, seed: int = 17) -> Path:
    """Writes the fixture checkpoint to `folder` (which must not exist)."""
    from transformers import LlamaConfig, LlamaForCausalLM

    folder = Path(folder)
    folder.mkdir(parents=True, exist_ok=False)
    torch.manual_seed(seed)
    config = LlamaConfig(**FIXTURE_CONFIG)
    LlamaForCausalLM(config).eval().save_pretrained(folder, safe_serialization=True)
    (folder / "fixture.json").write_text(json.dumps(
        {"kind": "synthetic-random-weights", "seed": seed, "purpose": "correctness only"},
        indent=2) + "\n")
    return folder


def state_digest(state: dict) -> str:
    """sha256 over sorted (name, raw bytes) of a state dict; identifies a checkpoint."""
    h = hashlib.sha256()
    for k in sorted(state):
        h.update(k.encode())
        h.update(state[k].contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


if __name__ == "__main__":
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--output", type=Path, required=True)
    parser.add_argument("--seed", type=int, default=17)
    options = parser.parse_args()
    create(options.output, options.seed)
