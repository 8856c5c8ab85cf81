"""hexgen2_b200: HexGen-2's disaggregated prefill/decode hot path, native to B200 (sm_100a).

Public API (mirrors the reference's):
    Engine, CacheState                     hexgen2/model.py
    GPTLMHeadModel, InferenceParams        hexgen/hexgen_core/models/gpt.py
    send_packet, recv_packet, send_data,
    recv_data, validate_header, KVHandoff  hexgen2/transport.py (+ the NVLink direct path)
The native engine's compute runs in libhexgen2_b200.so (see include/hexgen2_b200.h) and has
no CPU path; Engine(engine="hf-reference") is the reference's transformers-eager validation
engine, chosen explicitly, and runs none of it.
"""
from .engine import ContinuousBatcher, Engine, serve_arrivals
from .gpt import CacheState, GPTLMHeadModel, InferenceParams
from .transport import KVHandoff, recv_data, recv_packet, send_data, send_packet, validate_header

__all__ = ["Engine", "ContinuousBatcher", "serve_arrivals", "CacheState", "GPTLMHeadModel", "InferenceParams", "KVHandoff",
           "send_packet", "recv_packet", "send_data", "recv_data", "validate_header"]
