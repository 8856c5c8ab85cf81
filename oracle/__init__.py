"""Test infrastructure: CPU restatement of HexGen-2's prefill/decode hot path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import
this package, and only as the checker or the timed CPU baseline. The product path
(hexgen2_b200) never imports it and has no CPU fallback.
"""
