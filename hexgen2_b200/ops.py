"""Torch-facing wrappers over the C ABI: one function per kernel entry point.

Tensors are passed as raw device pointers plus sizes/strides; every launch goes on torch's
current CUDA stream. Scratch space (split-K partials, decode split partials) comes from a
per-device buffer that grows on demand and is reused across calls on the same stream.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import HX_EPI_NONE, HX_EPI_RESIDUAL, HX_EPI_SWIGLU, check  # noqa: F401

DTYPE_CODE = {torch.float32: _lib.HX_F32, torch.float16: _lib.HX_F16, torch.bfloat16: _lib.HX_BF16}


def _L():
    return _lib.lib()


def _code(t: torch.Tensor) -> int:
    try:
        return DTYPE_CODE[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}") from None


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("hexgen2_b200 kernels take CUDA tensors (there is no CPU path)")


_workspaces: dict[int, torch.Tensor] = {}

# Number of kernels launched through this module (bench.py reports it as gpu_launches; a CUDA
# graph replay adds the launches it captured).
LAUNCHES = 0
# Bumped whenever a scratch buffer is reallocated: CUDA graphs that captured the old address
# must not be replayed.
WORKSPACE_GEN = 0


def _count(launches=1):
    global LAUNCHES
    LAUNCHES += launches


def workspace(nbytes: int, device=None, kind: str = "attn") -> torch.Tensor | None:
    """Per-device scratch buffer of at least nbytes (None for 0), one per kind, reused across
    calls on the same stream (GEMM split-K partials, decode-attention split partials)."""
    if nbytes == 0:
        return None
    dev = torch.cuda.current_device() if device is None else torch.device(device).index
    key = (dev, kind)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        global WORKSPACE_GEN
        size = max(nbytes, 0 if buf is None else buf.numel() * 2)
        buf = torch.empty(size, dtype=torch.uint8, device=f"cuda:{dev}")
        _workspaces[key] = buf
        WORKSPACE_GEN += 1
    return buf


# ----------------------------------------------------------------------------- norms
def rmsnorm(x, weight, eps, add=None, residual_out=None, out=None, rows=None, in_stride=None):
    """out = RMSNorm(x (+ add)) * weight, residual_out = x (+ add); rows of x at in_stride."""
    _require_cuda(x, weight, add)
    hidden = weight.shape[0]
    if rows is None:
        rows = x.numel() // hidden
    if in_stride is None:
        in_stride = x.stride(-2) if x.dim() >= 2 else hidden
    if out is None:
        out = torch.empty(rows, hidden, dtype=x.dtype, device=x.device)
    check(_L().hx_rmsnorm(_p(x), _p(add), _p(residual_out), _p(out), _p(weight), rows, hidden,
                          in_stride, out.stride(-2) if out.dim() >= 2 else hidden, float(eps),
                          _code(x), _stream()), "hx_rmsnorm")
    _count(1)
    return out


def embed_rmsnorm(ids, table, weight, eps, residual_out, normed_out):
    _require_cuda(ids, table)
    check(_L().hx_embed_rmsnorm(_p(ids), ids.numel(), _p(table), table.shape[1], _p(weight),
                                float(eps), _p(residual_out), _p(normed_out), _code(table),
                                _stream()), "hx_embed_rmsnorm")
    _count(1)


def embedding(ids, table, vocab_start=0, out=None):
    _require_cuda(ids, table)
    hidden = table.shape[1]
    if out is None:
        out = torch.empty(ids.numel(), hidden, dtype=table.dtype, device=table.device)
    check(_L().hx_embedding(_p(ids), ids.numel(), _p(table), vocab_start, table.shape[0], hidden,
                            _p(out), _code(table), _stream()), "hx_embedding")
    _count(1)
    return out


# ----------------------------------------------------------------------------- rotary
def rotary_cache_write(qkv, batch, seqlen, n_heads, n_heads_kv, head_dim, pos_start, cos, sin,
                       cache, q_out=None, batch_offset=0, interleaved=True):
    """Rotates q/k of the packed qkv and writes k/v into cache [B, S_max, 2, hkv, d]."""
    _require_cuda(qkv, cache, pos_start)
    if q_out is None:
        q_out = torch.empty(batch, seqlen, n_heads, head_dim, dtype=qkv.dtype, device=qkv.device)
    assert cache.stride(-1) == 1 and cache.stride(-2) == head_dim and cache.stride(-3) == n_heads_kv * head_dim
    check(_L().hx_rotary_cache_write(_p(qkv), batch, seqlen, n_heads, n_heads_kv, head_dim,
                                     _p(pos_start), _p(cos), _p(sin), cos.shape[0],
                                     1 if interleaved else 0, _p(q_out), _p(cache),
                                     cache.stride(0), cache.stride(1), batch_offset,
                                     cache.shape[1], _code(qkv), _stream()),
          "hx_rotary_cache_write")
    _count(1)
    return q_out


# ----------------------------------------------------------------------------- gemm
def gemm(a, w, epilogue=HX_EPI_NONE, residual=None, out=None):
    """out = a @ w.T with an epilogue; a [M, K] (row-strided), w [N, K]."""
    _require_cuda(a, w, residual)
    M, K = a.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"gemm: shape mismatch {tuple(a.shape)} x {tuple(w.shape)}^T")
    n_out = N // 2 if epilogue == HX_EPI_SWIGLU else N
    if out is None:
        out = torch.empty(M, n_out, dtype=a.dtype, device=a.device)
    code = _code(a)
    nbytes = _L().hx_gemm_workspace(M, N, K, epilogue, code)
    ws = workspace(nbytes, kind="gemm" if code != _lib.HX_F32 else "attn")
    check(_L().hx_gemm(_p(a), _p(w), _p(out), M, N, K, a.stride(0), w.stride(0), out.stride(0),
                       epilogue, _p(residual), residual.stride(0) if residual is not None else 0,
                       _p(ws), nbytes, code, _stream()), "hx_gemm")
    _count(2 if nbytes else 1)
    return out


def gemm_qkv_rotary(x, w_qkv, seqlen, n_heads, n_heads_kv, head_dim, pos_start, cos, sin,
                    cache, q_out=None, batch_offset=0):
    """Wqkv GEMM with rotary + KV-cache write fused into its epilogue (f16/bf16): returns q
    [rows, n_heads, head_dim]; k, v land in cache[batch_offset + b, pos_start[b] + s]."""
    _require_cuda(x, w_qkv, cache, pos_start)
    M, K = x.shape
    N = w_qkv.shape[0]
    if q_out is None:
        q_out = torch.empty(M, n_heads, head_dim, dtype=x.dtype, device=x.device)
    code = _code(x)
    nbytes = _L().hx_gemm_workspace(M, N, K, _lib.HX_EPI_QKV_ROTARY, code)
    ws = workspace(nbytes, kind="gemm")
    check(_L().hx_gemm_qkv_rotary(_p(x), _p(w_qkv), M, K, x.stride(0), seqlen, n_heads,
                                  n_heads_kv, head_dim, _p(pos_start), _p(cos), _p(sin),
                                  cos.shape[0], _p(q_out), _p(cache), cache.stride(0),
                                  cache.stride(1), batch_offset, cache.shape[1], _p(ws), nbytes,
                                  code, _stream()), "hx_gemm_qkv_rotary")
    _count(2 if (nbytes and M > 64) else 1)
    return q_out


def gemm_qkv_rotary_varlen(x, w_qkv, lengths, slots, n_heads, n_heads_kv, head_dim, cos, sin,
                           cache, q_out, meta=None):
    """gemm_qkv_rotary over prompts packed row after row in x [T, K] (prompt b: lengths[b]
    rows, cache row slots[b], positions from 0): q into q_out [T, n_heads, head_dim], k and v
    into cache[slots[b], s]. meta: a varlen_meta table (the same one prefill_attention_varlen
    reads; built here when omitted)."""
    _require_cuda(x, w_qkv, cache, q_out)
    M, K = x.shape
    N = w_qkv.shape[0]
    n = len(lengths)
    table, _, _ = meta if meta is not None else varlen_meta(lengths, slots, x.device)
    base = table.data_ptr()
    code = _code(x)
    nbytes = _L().hx_gemm_workspace(M, N, K, _lib.HX_EPI_QKV_ROTARY, code)
    ws = workspace(nbytes, kind="gemm")
    check(_L().hx_gemm_qkv_rotary_varlen(
        _p(x), _p(w_qkv), M, K, x.stride(0), base, base + 4 * (n + 1), base + 4 * (2 * n + 1), n,
        n_heads, n_heads_kv, head_dim, _p(cos), _p(sin), cos.shape[0], _p(q_out), _p(cache),
        cache.stride(0), cache.stride(1), cache.shape[0], cache.shape[1], _p(ws), nbytes, code,
        _stream()), "hx_gemm_qkv_rotary_varlen")
    _count(2 if (nbytes and M > 64) else 1)
    return q_out


def gemm_workspace_bytes(M, N, K, epilogue, dtype) -> int:
    return _L().hx_gemm_workspace(M, N, K, epilogue, DTYPE_CODE[dtype])


# ----------------------------------------------------------------------------- attention
def prefill_attention(q, cache, pos_start, n_heads_kv, softmax_scale, causal=True, out=None,
                      batch_offset=0):
    """q [B, S, hq, d] against cache[batch_offset + b, :pos_start[b] + S]."""
    _require_cuda(q, cache, pos_start)
    B, S, hq, d = q.shape
    if out is None:
        out = torch.empty_like(q)
    check(_L().hx_prefill_attention(_p(q), _p(cache), cache.stride(0), cache.stride(1),
                                    batch_offset, _p(pos_start), B, S, hq, n_heads_kv, d,
                                    1 if causal else 0, float(softmax_scale), _p(out), _code(q),
                                    _stream()), "hx_prefill_attention")
    _count(1)
    return out


def varlen_table(lengths, slots):
    """Host layout of a packed pass's metadata, as int32 values: row offsets [n + 1], cache
    slots [n], start positions [n] (0: prefill from an empty cache), a pad to an even count, then
    the (prompt, 128-query block) work items, heaviest causal work (latest block) first.
    Returns (values, n_items, index of the first item)."""
    n = len(lengths)
    if n == 0 or len(slots) != n or any(L <= 0 for L in lengths):
        raise ValueError("varlen_table needs one slot and a positive length per prompt")
    offs = [0]
    for L in lengths:
        offs.append(offs[-1] + L)
    items = sorted(((b, qb) for b, L in enumerate(lengths) for qb in range(-(-L // 128))),
                   key=lambda it: (-it[1], it[0]))
    head = offs + list(slots) + [0] * n
    if len(head) % 2:
        head.append(0)  # the (prompt, block) pairs are read as 8-byte int2
    return head + [v for it in items for v in it], len(items), len(head)


def varlen_meta(lengths, slots, device):
    """varlen_table on the device (pinned host copy, asynchronous H2D on the current stream):
    the table prefill_attention_varlen and gemm_qkv_rotary_varlen read. Returns (table,
    n_items, items start index)."""
    values, n_items, items_at = varlen_table(lengths, slots)
    meta = torch.tensor(values, dtype=torch.int32).pin_memory()
    return meta.to(device, non_blocking=True), n_items, items_at


def prefill_attention_varlen(q, cache, lengths, slots, n_heads_kv, softmax_scale, out,
                             meta=None) -> bool:
    """Causal prefill attention of several prompts packed row after row in q [T, hq, d] (prompt
    b: lengths[b] rows, cache row slots[b], positions from 0) in ONE launch, into out. meta: a
    varlen_meta table (built here when omitted; build it beforehand for a CUDA-graph capture).
    Returns False, launching nothing, for shapes the tensor-core kernel does not cover (f32,
    head_dim 32); the caller then attends prompt by prompt."""
    _require_cuda(q, cache, out)
    T, hq, d = q.shape
    n = len(lengths)
    table, n_items, items_at = meta if meta is not None else varlen_meta(lengths, slots, q.device)
    base = table.data_ptr()
    st = _L().hx_prefill_attention_varlen(
        _p(q), _p(cache), cache.stride(0), cache.stride(1), cache.shape[0], base,
        base + 4 * (n + 1), base + 4 * (2 * n + 1), base + 4 * items_at, n, n_items, T, hq,
        n_heads_kv, d, 1, float(softmax_scale), _p(out), _code(q), _stream())
    if st == _lib.HX_ERR_UNSUPPORTED:
        return False
    check(st, "hx_prefill_attention_varlen")
    _count(1)
    return True


def decode_attention(q, cache, seqlens, n_heads_kv, max_seqlen, softmax_scale, out=None):
    """q [B, hq, d] against cache[b, :seqlens[b]] (seqlens int32 on device)."""
    _require_cuda(q, cache, seqlens)
    B, hq, d = q.shape[0], q.shape[-2], q.shape[-1]
    if out is None:
        out = torch.empty(B, hq, d, dtype=q.dtype, device=q.device)
    nbytes = _L().hx_decode_attention_workspace(B, hq, d, max_seqlen)
    ws = workspace(nbytes)
    check(_L().hx_decode_attention(_p(q), _p(cache), cache.stride(0), cache.stride(1),
                                   _p(seqlens), B, hq, n_heads_kv, d, max_seqlen,
                                   float(softmax_scale), _p(out), _p(ws), nbytes, _code(q),
                                   _stream()), "hx_decode_attention")
    _count(2 if nbytes else 1)
    return out


def decode_workspace_bytes(batch, n_heads, head_dim, max_seqlen) -> int:
    return _L().hx_decode_attention_workspace(batch, n_heads, head_dim, max_seqlen)


# ----------------------------------------------------------------------------- sampling
def argmax(logits, out=None):
    _require_cuda(logits)
    rows, cols = logits.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.long, device=logits.device)
    check(_L().hx_argmax(_p(logits), rows, cols, logits.stride(0), _p(out), _code(logits),
                         _stream()), "hx_argmax")
    _count(1)
    return out


# ----------------------------------------------------------------------------- KV handoff
def kv_pack(src_ptrs, live_rows, dst_offsets, n_outer, outer_stride_bytes, row_stride_bytes,
            row_bytes, max_live_rows, dst):
    """Gather-pack of live rows (see hx_kv_pack). Pointer/length/offset arrays are int64 CUDA
    tensors; dst may be a peer GPU's buffer given as a raw address (int)."""
    dst_ptr = dst if isinstance(dst, int) else dst.data_ptr()
    check(_L().hx_kv_pack(_p(src_ptrs), _p(live_rows), _p(dst_offsets), src_ptrs.numel(),
                          n_outer, outer_stride_bytes, row_stride_bytes, row_bytes,
                          max_live_rows, dst_ptr, _stream()), "hx_kv_pack")
    _count(1)


def kv_unpack(src, src_offsets, live_rows, dst_ptrs, n_outer, outer_stride_bytes,
              row_stride_bytes, row_bytes, max_live_rows):
    src_ptr = src if isinstance(src, int) else src.data_ptr()
    check(_L().hx_kv_unpack(src_ptr, _p(src_offsets), _p(live_rows), _p(dst_ptrs),
                            dst_ptrs.numel(), n_outer, outer_stride_bytes, row_stride_bytes,
                            row_bytes, max_live_rows, _stream()), "hx_kv_unpack")
    _count(1)


def device_error(clear=True) -> int:
    return _L().hx_device_error(1 if clear else 0)
