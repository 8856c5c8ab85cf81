"""hx_decode_attention_noalloc: decode attention for callers that cannot allocate device memory
(a host runtime with a fixed, pre-carved device-memory budget, or a latency-critical loop
where a possibly synchronising cudaMalloc is not allowed). Its split partials live in a static
device array instead of a caller-provided workspace. Called here through the C ABI, twice in a
row, and compared with the workspace entry point hx_decode_attention on the same inputs and
with the CPU oracle's FlashAttention-numerics attention (oracle/llama_ref.py flash_attention).
The cases cover both partial layouts that land in the static array: the balanced TMA kernels
(bf16, head_dim 64/128) and the fixed-split kernels (head_dim 32, and f32).

This file is named so pytest collects it last; it passes alone in a fresh process and after
the rest of the suite.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 << 20  # HX_DECODE_NOALLOC_SCRATCH_BYTES in include/hexgen2_b200.h
CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}  # HX_F32, HX_F16, HX_BF16
TOL = {torch.bfloat16: 2e-2, torch.float32: 1e-4}


def _call(lib, fn, q, cache, seqlens, hk, max_len, scale, out, ws=None):
    B, hq, d = q.shape
    code = CODES[q.dtype]
    stream = torch.cuda.current_stream().cuda_stream
    if fn == "noalloc":
        return lib.hx_decode_attention_noalloc(q.data_ptr(), cache.data_ptr(), cache.stride(0),
                                               cache.stride(1), seqlens.data_ptr(), B, hq, hk, d,
                                               max_len, scale, out.data_ptr(), code, stream)
    nbytes = lib.hx_decode_attention_workspace(B, hq, d, max_len)
    return lib.hx_decode_attention(q.data_ptr(), cache.data_ptr(), cache.stride(0), cache.stride(1),
                                   seqlens.data_ptr(), B, hq, hk, d, max_len, scale, out.data_ptr(),
                                   None if ws is None else ws.data_ptr(), nbytes, code, stream)


@pytest.mark.parametrize("B,hq,hk,d,lens,dtype", [
    (2, 8, 2, 128, [3000, 17], torch.bfloat16),        # balanced TMA kernel, 4 heads per group
    (1, 32, 32, 128, [1200], torch.bfloat16),          # balanced TMA kernel, MHA
    (4, 32, 4, 64, [1, 64, 65, 700], torch.bfloat16),  # tensor-core grouped kernel
    (3, 8, 2, 32, [5, 300, 1000], torch.bfloat16),     # fixed-split kernel (head_dim 32)
    (2, 8, 8, 128, [900, 33], torch.float32),          # fixed-split kernel (f32)
])
def test_noalloc_matches_workspace_entry_point(B, hq, hk, d, lens, dtype):
    from hexgen2_b200 import _lib
    from oracle.llama_ref import flash_attention
    lib = _lib.lib()
    g = torch.Generator().manual_seed(B * 100 + d)
    cap = max(lens) + 5
    q_h = torch.randn(B, hq, d, generator=g).to(dtype)
    cache_h = torch.randn(B, cap, 2, hk, d, generator=g).to(dtype)
    q, cache = q_h.cuda(), cache_h.cuda()
    seqlens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    scale = d ** -0.5
    tol = TOL[dtype]
    nbytes = lib.hx_decode_attention_workspace(B, hq, d, cap)
    assert 0 < nbytes <= SCRATCH_BYTES  # these shapes use split scratch
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    ref = torch.empty(B, hq, d, dtype=dtype, device="cuda")
    assert _call(lib, "workspace", q, cache, seqlens, hk, cap, scale, ref, ws) == 0
    oracle = torch.cat([flash_attention(q_h[b:b + 1, None], cache_h[b:b + 1, :L], False, scale)[:, 0]
                        for b, L in enumerate(lens)])
    for _ in range(2):  # two calls in a row share (and reuse) the static scratch
        out = torch.full_like(ref, float("nan"))
        assert _call(lib, "noalloc", q, cache, seqlens, hk, cap, scale, out) == 0, \
            lib.hx_last_error().decode()
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref.float(), rtol=tol, atol=tol)
        torch.testing.assert_close(out.float().cpu(), oracle.float(), rtol=tol, atol=tol)
    assert lib.hx_device_error(1) == 0


def test_noalloc_rejects_shapes_beyond_the_static_scratch():
    from hexgen2_b200 import _lib
    lib = _lib.lib()
    checked = 0
    # The first shape needs ~19 MiB of split partials (592 splits of an
    # 8192-wide head); the others are large serving shapes.
    for B, hq, d, L in [(1, 1, 8192, 65536), (64, 64, 128, 65536), (256, 64, 128, 32768)]:
        need = lib.hx_decode_attention_workspace(B, hq, d, L)
        if need <= SCRATCH_BYTES:
            continue
        checked += 1
        q = torch.zeros(1, dtype=torch.bfloat16, device="cuda")  # never read: rejected first
        rc = lib.hx_decode_attention_noalloc(q.data_ptr(), q.data_ptr(), 2 * hq * d * L,
                                             2 * hq * d, q.data_ptr(), B, hq, hq, d, L, 0.1,
                                             q.data_ptr(), CODES[torch.bfloat16],
                                             torch.cuda.current_stream().cuda_stream)
        assert rc == _lib.HX_ERR_INVALID
        assert b"static array" in lib.hx_last_error()
    assert checked >= 1
