"""Kernel-level parity on the GPU: every C-ABI entry point against the CPU oracle (or an f32
torch reference with the same rounding points) on the same seeded inputs."""
import pytest
import torch

from oracle.llama_ref import Rotary, flash_attention, rms_norm
from tests.conftest import from_bits

pytestmark = pytest.mark.gpu

DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


@pytest.fixture(scope="module")
def ops():
    from hexgen2_b200 import ops as o
    return o


def ulp_tol(dtype):
    return {torch.bfloat16: 2 ** -7, torch.float16: 2 ** -10, torch.float32: 1e-5}[dtype]


# ------------------------------------------------------------------------------ rmsnorm
@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("hidden", [128, 100, 2048, 4096, 8192])
@pytest.mark.parametrize("with_add", [False, True])
def test_rmsnorm(ops, dtype, hidden, with_add):
    dt = DT[dtype]
    g = torch.Generator().manual_seed(hidden)
    x = torch.randn(37, hidden, generator=g).to(dt)
    add = torch.randn(37, hidden, generator=g).to(dt) if with_add else None
    w = (torch.rand(hidden, generator=g) + 0.5).to(dt)
    res_ref = (x + add) if with_add else x
    ref = rms_norm(res_ref, w, 1e-5)
    res = torch.empty(37, hidden, dtype=dt, device="cuda")
    out = ops.rmsnorm(x.cuda(), w.cuda(), 1e-5, add=None if add is None else add.cuda(),
                      residual_out=res)
    torch.testing.assert_close(res.cpu(), res_ref, rtol=0, atol=0)
    # Sum order / rsqrt rounding may flip the last bit of a few elements.
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=2 * ulp_tol(dt), atol=1e-6)
    if dt != torch.float32:  # in f32 a 1-ulp rstd difference moves every element
        exact = (out.cpu() == ref).float().mean().item()
        assert exact > 0.97, exact


def test_rmsnorm_matches_reference_kat(ops, golden):
    for row in golden["rmsnorm"]:
        dt = {"torch.float32": torch.float32, "torch.float16": torch.float16,
              "torch.bfloat16": torch.bfloat16}[row["dtype"]]
        x = from_bits(row["input"], dt).reshape(7, 128)
        w = from_bits(row["weight"], dt)
        out = ops.rmsnorm(x.cuda(), w.cuda(), row["eps"]).cpu().flatten()
        expected = from_bits(row["output"], dt)
        torch.testing.assert_close(out.float(), expected.float(), rtol=2 * ulp_tol(dt), atol=1e-6)


def test_embed_rmsnorm(ops):
    g = torch.Generator().manual_seed(3)
    table = torch.randn(500, 256, generator=g).bfloat16()
    w = (torch.rand(256, generator=g) + 0.5).bfloat16()
    ids = torch.randint(0, 500, (19,), generator=g)
    res = torch.empty(19, 256, dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(res)
    ops.embed_rmsnorm(ids.cuda(), table.cuda(), w.cuda(), 1e-6, res, out)
    torch.testing.assert_close(res.cpu(), table[ids], rtol=0, atol=0)
    torch.testing.assert_close(out.cpu().float(), rms_norm(table[ids], w, 1e-6).float(),
                               rtol=2 ** -6, atol=1e-6)


def test_vocab_parallel_embedding(ops):
    table = torch.randn(64, 32).bfloat16()
    ids = torch.tensor([0, 5, 31, 32, 40, 63])
    out = ops.embedding(ids.cuda(), table[32:].cuda(), vocab_start=32).cpu()
    ref = table[ids].clone()
    ref[ids < 32] = 0
    torch.testing.assert_close(out, ref, rtol=0, atol=0)


# ------------------------------------------------------------------------------ gemm
def gemm_ref(a, b, epi, res, dt):
    acc = a.float() @ b.float().T
    if epi == 0:
        return acc.to(dt)
    if epi == 1:
        return (acc.to(dt).float() + res.float()).to(dt)
    n = acc.shape[1] // 2
    blocks = acc.view(acc.shape[0], n // 16, 2, 16)
    up = blocks[:, :, 0].reshape(acc.shape[0], n).to(dt).float()
    gate = blocks[:, :, 1].reshape(acc.shape[0], n).to(dt).float()
    silu = (gate / (1 + torch.exp(-gate))).to(dt).float()
    return (up * silu).to(dt)


GEMM_SHAPES = [(1, 64, 64), (7, 128, 128), (128, 256, 128), (129, 192, 256), (300, 2560, 2048),
               (1, 4096, 4096), (8, 4096, 11008), (32, 12288, 4096), (512, 2560, 2048),
               (1024, 1024, 1024), (64, 32000, 2048), (16, 12288, 4096), (48, 4096, 4096),
               (33, 22016, 4096), (65, 4096, 4096), (17, 100, 64)]


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_tcgen05(ops, dtype, M, N, K):
    dt = DT[dtype]
    g = torch.Generator().manual_seed(M * 7 + N * 3 + K)
    a = torch.randn(M, K, generator=g).to(dt)
    b = (torch.randn(N, K, generator=g) * 0.05).to(dt)
    out = ops.gemm(a.cuda(), b.cuda()).cpu()
    ref = gemm_ref(a, b, 0, None, dt)
    torch.testing.assert_close(out.float(), ref.float(), rtol=2 * ulp_tol(dt), atol=1e-3)


@pytest.mark.parametrize("M,N,K", [(5, 256, 128), (300, 512, 2048), (1, 22016, 4096), (77, 11264, 2048),
                                   (37, 4096, 11008), (32, 4096, 4096), (64, 22016, 4096)])
def test_gemm_epilogues(ops, M, N, K):
    dt = torch.bfloat16
    g = torch.Generator().manual_seed(N + K)
    a = torch.randn(M, K, generator=g).to(dt)
    b = (torch.randn(N, K, generator=g) * 0.05).to(dt)
    res = torch.randn(M, N, generator=g).to(dt)
    out = ops.gemm(a.cuda(), b.cuda(), ops.HX_EPI_RESIDUAL, residual=res.cuda()).cpu()
    torch.testing.assert_close(out.float(), gemm_ref(a, b, 1, res, dt).float(), rtol=2 ** -6, atol=2e-2)
    out = ops.gemm(a.cuda(), b.cuda(), ops.HX_EPI_SWIGLU).cpu()
    # SwiGLU rounds four times (up, gate, silu(gate), product), so a 1-ulp f32-order flip in the
    # accumulator can surface as a few ulps of the output: 4 bf16 ulps relative.
    torch.testing.assert_close(out.float(), gemm_ref(a, b, 2, None, dt).float(), rtol=2 ** -5, atol=2e-3)
    # In-place residual (the model updates the residual stream in place).
    r = res.cuda().clone()
    ops.gemm(a.cuda(), b.cuda(), ops.HX_EPI_RESIDUAL, residual=r, out=r)
    torch.testing.assert_close(r.cpu().float(), gemm_ref(a, b, 1, res, dt).float(), rtol=2 ** -6, atol=2e-2)


# Shapes that run on CTA pairs (256 x 256 tiles over two SMs): M tails that leave the odd CTA's
# rows wholly out of range (300, 257), an N tail that does the same for its columns (16000),
# long K, the model's projection shapes at a 900-token prompt, and partly filled waves (48 and
# 32 items on 74 pairs).
PAIR_SHAPES = [(900, 4096, 4096), (1000, 12288, 1024), (300, 22016, 512), (257, 16000, 256),
               (900, 4096, 11008), (640, 8192, 520), (700, 4096, 2048), (285, 4096, 1024)]


@pytest.mark.parametrize("M,N,K", PAIR_SHAPES)
def test_gemm_cta_pairs(ops, M, N, K):
    from hexgen2_b200 import _lib
    assert _lib.lib().hx_gemm_kernel_kind(M, N, K, _lib.HX_BF16) == 2
    dt = torch.bfloat16
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g).to(dt)
    b = (torch.randn(N, K, generator=g) * 0.05).to(dt)
    res = torch.randn(M, N, generator=g).to(dt)
    out = ops.gemm(a.cuda(), b.cuda()).cpu()
    torch.testing.assert_close(out.float(), gemm_ref(a, b, 0, None, dt).float(), rtol=2 * ulp_tol(dt), atol=1e-3)
    out = ops.gemm(a.cuda(), b.cuda(), ops.HX_EPI_RESIDUAL, residual=res.cuda()).cpu()
    # round(round(acc) + r): a summation-order flip of the inner rounding moves the result by
    # one ulp of acc, which the residual add does not shrink, so bound by both ulps.
    ref = gemm_ref(a, b, 1, res, dt).float()
    acc = a.float() @ b.float().T
    bound = acc.abs() * 2 ** -7 + ref.abs() * 2 ** -7 + 1e-3
    assert ((out.float() - ref).abs() <= bound).all(), (out.float() - ref).abs().max()
    out = ops.gemm(a.cuda(), b.cuda(), ops.HX_EPI_SWIGLU).cpu()
    torch.testing.assert_close(out.float(), gemm_ref(a, b, 2, None, dt).float(), rtol=2 ** -5, atol=2e-3)
    assert ops.device_error() == 0


@pytest.mark.parametrize("epi", [0, 1, 2])
def test_gemm_f32(ops, epi):
    g = torch.Generator().manual_seed(epi)
    a = torch.randn(33, 96, generator=g)
    b = torch.randn(64, 96, generator=g)
    res = torch.randn(33, 64, generator=g)
    out = ops.gemm(a.cuda(), b.cuda(), epi, residual=res.cuda() if epi == 1 else None).cpu()
    torch.testing.assert_close(out, gemm_ref(a, b, epi, res, torch.float32), rtol=1e-5, atol=1e-5)


def test_gemm_strided_rows(ops):
    """A operand given as a row-strided view (last-token rows of a [B, S, h] tensor)."""
    x = torch.randn(4, 9, 256).bfloat16().cuda()
    w = (torch.randn(512, 256) * 0.05).bfloat16().cuda()
    out = ops.gemm(x[:, -1], w)
    ref = gemm_ref(x[:, -1].cpu(), w.cpu(), 0, None, torch.bfloat16)
    torch.testing.assert_close(out.cpu().float(), ref.float(), rtol=2 ** -6, atol=1e-3)


# ------------------------------------------------------------------------------ rotary
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("hq,hk,d", [(4, 2, 32), (32, 4, 64), (32, 32, 128)])
def test_rotary_cache_write(ops, dtype, hq, hk, d):
    dt = DT[dtype]
    B, S, cap = 2, 13, 40
    g = torch.Generator().manual_seed(d)
    qkv = torch.randn(B, S, (hq + 2 * hk) * d, generator=g).to(dt)
    starts = torch.tensor([0, 11], dtype=torch.int32)
    rot = Rotary(d, 10000.0)
    cos, sin = rot.tables(64, dt)
    cache = torch.zeros(3, cap, 2, hk, d, dtype=dt, device="cuda")
    q = ops.rotary_cache_write(qkv.cuda(), B, S, hq, hk, d, starts.cuda(), cos.cuda(), sin.cuda(),
                               cache, batch_offset=1)
    for b in range(B):
        off = int(starts[b])
        qb = qkv[b:b + 1, :, : hq * d].reshape(1, S, hq, d)
        kv = qkv[b:b + 1, :, hq * d:].reshape(1, S, 2, hk, d)
        tol = dict(rtol=2 * ulp_tol(dt), atol=1e-6)
        torch.testing.assert_close(q[b].cpu().float(), rot.apply(qb, off, dt)[0].float(), **tol)
        torch.testing.assert_close(cache[1 + b, off:off + S, 0].cpu().float(),
                                   rot.apply(kv[:, :, 0], off, dt)[0].float(), **tol)
        torch.testing.assert_close(cache[1 + b, off:off + S, 1].cpu(), kv[0, :, 1], rtol=0, atol=0)
    assert cache[0].abs().sum().item() == 0  # other batch rows untouched


# ------------------------------------------------------------------------------ attention
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("hq,hk,d", [(4, 2, 32), (32, 4, 64), (32, 32, 128), (8, 1, 128)])
@pytest.mark.parametrize("S", [1, 7, 64, 129])
def test_prefill_attention(ops, dtype, hq, hk, d, S):
    dt = DT[dtype]
    g = torch.Generator().manual_seed(S * d + hq)
    B, cap = 2, 160
    q = torch.randn(B, S, hq, d, generator=g).to(dt)
    cache = torch.randn(B, cap, 2, hk, d, generator=g).to(dt)
    starts = torch.zeros(B, dtype=torch.int32)
    out = ops.prefill_attention(q.cuda(), cache.cuda(), starts.cuda(), hk, d ** -0.5).cpu()
    ref = flash_attention(q, cache[:, :S], True, d ** -0.5)
    tol = 2e-2 if dt != torch.float32 else 1e-5
    torch.testing.assert_close(out.float(), ref.float(), rtol=tol, atol=tol)


@pytest.mark.parametrize("d", [64, 128])
def test_prefill_attention_growing_scores(ops, d):
    """Scores that grow along the keys by far more than 2^8 per tile, so the tensor-core
    kernel must rescale its TMEM output several times per row; plus a long multi-block case
    with a start offset."""
    dt, hq, hk = torch.bfloat16, 4, 2
    g = torch.Generator().manual_seed(d)
    for B, S, start in ((1, 520, 0), (2, 300, 37)):
        cap = start + S + 3
        q = (torch.randn(B, S, hq, d, generator=g) * 2).to(dt)
        cache = torch.randn(B, cap, 2, hk, d, generator=g)
        ramp = 1 + 6 * torch.arange(cap, dtype=torch.float32) / cap
        cache[:, :, 0] *= ramp.view(1, cap, 1, 1)
        cache = cache.to(dt)
        starts = torch.full((B,), start, dtype=torch.int32)
        out = ops.prefill_attention(q.cuda(), cache.cuda(), starts.cuda(), hk, d ** -0.5).cpu()
        ref = flash_attention(q, cache[:, :start + S], True, d ** -0.5)
        torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)


def test_prefill_attention_offsets_and_noncausal(ops):
    dt, hq, hk, d = torch.bfloat16, 8, 2, 64
    g = torch.Generator().manual_seed(11)
    cache = torch.randn(2, 100, 2, hk, d, generator=g).to(dt)
    q = torch.randn(2, 5, hq, d, generator=g).to(dt)
    starts = torch.tensor([20, 70], dtype=torch.int32)
    for causal in (True, False):
        out = ops.prefill_attention(q.cuda(), cache.cuda(), starts.cuda(), hk, d ** -0.5,
                                    causal=causal).cpu()
        for b in range(2):
            n = int(starts[b]) + 5
            ref = flash_attention(q[b:b + 1], cache[b:b + 1, :n], causal, d ** -0.5)
            torch.testing.assert_close(out[b:b + 1].float(), ref.float(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("hq,hk,d", [(4, 2, 32), (32, 4, 64), (32, 32, 128), (64, 8, 128)])
@pytest.mark.parametrize("lens", [[1], [5, 64, 65], [1000, 3], [4095, 2048, 17, 1]])
def test_decode_attention(ops, dtype, hq, hk, d, lens):
    dt = DT[dtype]
    B, cap = len(lens), max(lens) + 3
    g = torch.Generator().manual_seed(sum(lens) + d)
    q = torch.randn(B, hq, d, generator=g).to(dt)
    cache = torch.randn(B, cap, 2, hk, d, generator=g).to(dt)
    seq = torch.tensor(lens, dtype=torch.int32)
    out = ops.decode_attention(q.cuda(), cache.cuda(), seq.cuda(), hk, cap, d ** -0.5).cpu()
    tol = 2e-2 if dt != torch.float32 else 1e-5
    for b, L in enumerate(lens):
        ref = flash_attention(q[b:b + 1, None], cache[b:b + 1, :L], False, d ** -0.5)[:, 0]
        torch.testing.assert_close(out[b:b + 1].float(), ref.float(), rtol=tol, atol=tol)


@pytest.mark.parametrize("hq,hk,d,lens", [(32, 32, 128, [300]), (64, 8, 128, [1000, 3]),
                                          (16, 2, 128, [700, 5, 260]), (32, 4, 64, [513])])
def test_decode_attention_few_tiles_stale_workspace(ops, hq, hk, d, lens):
    """Fewer 128-key tiles than SMs leave some CTAs without work; the merge of runs cut across
    CTAs must not read their (never written) partial slots. The scratch is filled with NaN
    first so a stale slot would show."""
    dt = torch.bfloat16
    B, cap = len(lens), max(lens) + 3
    g = torch.Generator().manual_seed(sum(lens) + hq)
    q = torch.randn(B, hq, d, generator=g).to(dt)
    cache = torch.randn(B, cap, 2, hk, d, generator=g).to(dt)
    seq = torch.tensor(lens, dtype=torch.int32)
    nbytes = ops.decode_workspace_bytes(B, hq, d, cap)
    ops.workspace(nbytes).view(torch.uint8).fill_(0xFF)  # NaN bit patterns everywhere
    out = ops.decode_attention(q.cuda(), cache.cuda(), seq.cuda(), hk, cap, d ** -0.5).cpu()
    assert torch.isfinite(out.float()).all()
    for b, L in enumerate(lens):
        ref = flash_attention(q[b:b + 1, None], cache[b:b + 1, :L], False, d ** -0.5)[:, 0]
        torch.testing.assert_close(out[b:b + 1].float(), ref.float(), rtol=2e-2, atol=2e-2)


# ------------------------------------------------------------------------------ KV re-shard
@pytest.mark.parametrize("src_tp,dst_tp", [(2, 4), (4, 2), (2, 1), (1, 8)])
def test_reshard_kv_matches_reference_head_concat(ops, src_tp, dst_tp):
    """Prefill TP != decode TP: the per-rank caches after the slice moves equal the reference's
    concat of the shards on the head dimension (tensor_parallel_dim_concat.py), split dst_tp
    ways. Bytes compared exactly."""
    from oracle.llama_ref import concat_kv_heads
    from hexgen2_b200.transport import reshard_kv
    layers, B, cap, H, d = 3, 3, 60, 8, 64
    lens = [17, 60, 1]
    rows = [2, 0, 1]  # request r lives in batch row rows[r]
    g = torch.Generator().manual_seed(src_tp * 10 + dst_tp)
    full = torch.randn(layers, B, cap, 2, H, d, generator=g).bfloat16()
    hs, hd = H // src_tp, H // dst_tp
    src = []
    for s in range(src_tp):
        shard = full[:, :, :, :, s * hs:(s + 1) * hs].contiguous().cuda()
        src.append({i: shard[i] for i in range(layers)})
    dst = []
    for t in range(dst_tp):
        big = torch.zeros(layers, B, cap, 2, hd, d, dtype=torch.bfloat16, device="cuda")
        dst.append({i: big[i] for i in range(layers)})
    reshard_kv(src, dst, rows, lens, H)
    torch.cuda.synchronize()
    for r, (row, L) in enumerate(zip(rows, lens)):
        shards = [{i: src[s][i][row:row + 1, :L].cpu() for i in range(layers)} for s in range(src_tp)]
        whole = concat_kv_heads(shards)
        for t in range(dst_tp):
            for i in range(layers):
                want = whole[i][..., t * hd:(t + 1) * hd, :]
                got = dst[t][i][row:row + 1, :L].cpu()
                assert torch.equal(got, want)
                # rows past the live length stay untouched
                assert not dst[t][i][row, L:].abs().sum().item()


# ------------------------------------------------------------------------------ argmax
@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("cols", [32000, 32003, 7])
def test_argmax_ties_first_index(ops, dtype, cols):
    dt = DT[dtype]
    x = torch.randn(7, cols).to(dt)
    x[1, 1] = x[1, cols - 2] = 50.0
    x[2, :] = 1.0
    x[3, cols - 1] = 99.0
    x[4, 3] = float("nan")  # NaN is the maximum, like torch.argmax
    out = ops.argmax(x.cuda()).cpu()
    assert out.tolist() == x.argmax(-1).tolist()
    assert out[2].item() == 0 and out[1].item() == 1 and out[4].item() == 3
    # Row-strided view whose rows start off a 16-byte boundary (scalar path).
    wide = torch.randn(7, cols + 1).to(dt)
    wide[:, 1:] = x
    got = ops.argmax(wide.cuda()[:, 1:]).cpu()
    assert got.tolist() == x.argmax(-1).tolist()


# ------------------------------------------------------------------------------ KV pack
def test_kv_pack_unpack_bit_exact(ops):
    g = torch.Generator().manual_seed(0)
    layers, cap, hk, d = 3, 50, 2, 32
    big = torch.randn(layers, 4, cap, 2, hk, d, generator=g).bfloat16().cuda()
    lens = [7, 0, 50, 1]
    rows = 2 * hk * d * 2
    offs, o = [], 0
    for L in lens:
        offs.append(o)
        o += layers * L * rows
    packed = torch.empty(max(o, 16), dtype=torch.uint8, device="cuda")
    elem = 2
    src = torch.tensor([big.data_ptr() + b * big.stride(1) * elem for b in range(4)], device="cuda")
    ops.kv_pack(src, torch.tensor(lens, device="cuda"), torch.tensor(offs, device="cuda"), layers,
                big.stride(0) * elem, big.stride(2) * elem, rows, max(lens), packed)
    for b, (L, off) in enumerate(zip(lens, offs)):
        got = packed[off:off + layers * L * rows].view(torch.bfloat16).view(layers, L, 2, hk, d)
        assert torch.equal(got.cpu(), big[:, b, :L].cpu())
    back = torch.zeros_like(big)
    dst = torch.tensor([back.data_ptr() + b * back.stride(1) * elem for b in range(4)], device="cuda")
    ops.kv_unpack(packed, torch.tensor(offs, device="cuda"), torch.tensor(lens, device="cuda"), dst,
                  layers, back.stride(0) * elem, back.stride(2) * elem, rows, max(lens))
    for b, L in enumerate(lens):
        assert torch.equal(back[:, b, :L].cpu(), big[:, b, :L].cpu())
        assert back[:, b, L:].abs().sum().item() == 0


def test_kv_pack_microbench_layout(ops):
    """[layers, 2, kv_heads, max_seq, head_dim] per request (the KV handoff microbenchmark)."""
    layers, hk, cap, d = 4, 8, 256, 128
    reqs = [torch.randn(layers, 2, hk, cap, d).bfloat16().cuda() for _ in range(3)]
    lens = [128, 256, 1]
    rb = d * 2
    offs, o = [], 0
    for L in lens:
        offs.append(o)
        o += layers * 2 * hk * L * rb
    packed = torch.empty(o, dtype=torch.uint8, device="cuda")
    ops.kv_pack(torch.tensor([r.data_ptr() for r in reqs], device="cuda"),
                torch.tensor(lens, device="cuda"), torch.tensor(offs, device="cuda"),
                layers * 2 * hk, cap * rb, rb, rb, max(lens), packed)
    for r, L, off in zip(reqs, lens, offs):
        got = packed[off:off + layers * 2 * hk * L * rb].view(torch.bfloat16).view(layers, 2, hk, L, d)
        assert torch.equal(got.cpu(), r[:, :, :, :L].cpu())


def test_errors_are_reported_not_crashes(ops):
    with pytest.raises(ValueError):
        ops.gemm(torch.randn(4, 8).bfloat16().cuda(), torch.randn(8, 16).bfloat16().cuda())
    with pytest.raises(NotImplementedError):
        q = torch.randn(1, 2, 48).bfloat16().cuda()
        ops.decode_attention(q, torch.zeros(1, 4, 2, 2, 48).bfloat16().cuda(),
                             torch.tensor([1], dtype=torch.int32, device="cuda"), 2, 4, 0.1)
    assert ops.device_error() == 0


# ------------------------------------------------------------------------------ fused Wqkv
@pytest.mark.parametrize("B,S,hq,hk,d", [(4, 1, 32, 32, 128), (32, 1, 32, 32, 128), (1, 300, 32, 4, 64),
                                         (2, 77, 8, 2, 128), (64, 1, 16, 2, 128), (3, 1, 4, 2, 32),
                                         (1, 1000, 32, 8, 128), (2, 450, 32, 32, 128)])
def test_gemm_qkv_rotary_matches_separate_path(ops, B, S, hq, hk, d):
    """Wqkv GEMM with rotary + cache write in its epilogue == GEMM, then hx_rotary_cache_write."""
    dt, h = torch.bfloat16, hq * d
    g = torch.Generator().manual_seed(B * 1000 + S)
    x = torch.randn(B * S, h, generator=g).to(dt).cuda()
    w = (torch.randn((hq + 2 * hk) * d, h, generator=g) * 0.05).to(dt).cuda()
    starts = torch.tensor([(7 * i) % 50 for i in range(B)], dtype=torch.int32).cuda()
    cap = 50 + S + 1
    cos, sin = Rotary(d, 10000.0).tables(cap + 1, dt)
    cos, sin = cos.cuda(), sin.cuda()
    c_ref = torch.zeros(B + 1, cap, 2, hk, d, dtype=dt, device="cuda")
    c_new = torch.zeros_like(c_ref)
    qkv = ops.gemm(x, w)
    q_ref = ops.rotary_cache_write(qkv, B, S, hq, hk, d, starts, cos, sin, c_ref, batch_offset=1)
    q_new = ops.gemm_qkv_rotary(x, w, S, hq, hk, d, starts, cos, sin, c_new, batch_offset=1)
    torch.testing.assert_close(q_new.view(B, S, hq, d).float(), q_ref.float(), rtol=2 ** -7, atol=1e-6)
    torch.testing.assert_close(c_new.float(), c_ref.float(), rtol=2 ** -7, atol=1e-6)
    assert ops.device_error() == 0


@pytest.mark.parametrize("M,N,K", [(32, 4096, 4096), (8, 12288, 4096), (64, 4096, 11008),
                                   (3, 2560, 2048), (17, 200, 4160)])
def test_decode_gemm_is_deterministic_and_needs_no_workspace(ops, M, N, K):
    """Decode-shaped GEMMs (M <= 64) split K inside a cluster and sum the partials in rank
    order: repeated calls are bit-identical and no scratch memory is requested."""
    from hexgen2_b200 import _lib
    dt = torch.bfloat16
    assert _lib.lib().hx_gemm_workspace(M, N, K, ops.HX_EPI_RESIDUAL, _lib.HX_BF16) == 0
    g = torch.Generator().manual_seed(M + N)
    a = torch.randn(M, K, generator=g).to(dt)
    b = (torch.randn(N, K, generator=g) * 0.05).to(dt)
    r = torch.randn(M, N, generator=g).to(dt)
    outs = [ops.gemm(a.cuda(), b.cuda(), ops.HX_EPI_RESIDUAL, residual=r.cuda()) for _ in range(3)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    torch.testing.assert_close(outs[0].cpu().float(), gemm_ref(a, b, 1, r, dt).float(),
                               rtol=2 ** -6, atol=2e-2)
    assert ops.device_error() == 0


# ------------------------------------------------------------------------------ varlen prefill
@pytest.mark.parametrize("lens,hq,hk,d", [([1, 17, 30], 8, 2, 128),          # M <= 64: decode kernel
                                          ([129, 1, 70], 8, 2, 128),         # split-K tcgen05 tiles
                                          ([5, 300, 77], 16, 2, 64),
                                          ([700, 1300, 1, 64], 32, 8, 128)])  # CTA-pair tiles
def test_gemm_qkv_rotary_varlen_matches_per_prompt(ops, lens, hq, hk, d):
    """Packed prompts through the Wqkv GEMM with rotary + cache write in its epilogue (each
    row rotated at its position within its prompt, k/v into the prompt's cache slot) == the
    plain GEMM followed by hx_rotary_cache_write prompt by prompt (within one bf16 ulp:
    the two kernels may contract the rotary's multiply-adds differently); slots not named stay
    untouched. A slot outside the cache is never written and is reported in the device
    error word."""
    dt, h = torch.bfloat16, hq * d
    n = len(lens)
    slots = [(3 * i + 1) % (n + 1) for i in range(n)]
    T, cap = sum(lens), max(lens) + 3
    g = torch.Generator().manual_seed(T + hq)
    x = torch.randn(T, h, generator=g).to(dt).cuda()
    w = (torch.randn((hq + 2 * hk) * d, h, generator=g) * 0.05).to(dt).cuda()
    cos, sin = Rotary(d, 10000.0).tables(cap, dt)
    cos, sin = cos.cuda(), sin.cuda()
    c_ref = torch.zeros(n + 1, cap, 2, hk, d, dtype=dt, device="cuda")
    c_new = torch.zeros_like(c_ref)
    qkv = ops.gemm(x, w)
    zero = torch.zeros(1, dtype=torch.int32, device="cuda")
    q_ref = torch.empty(T, hq, d, dtype=dt, device="cuda")
    o = 0
    for b, L in enumerate(lens):
        ops.rotary_cache_write(qkv[o:o + L], 1, L, hq, hk, d, zero, cos, sin, c_ref,
                               q_out=q_ref[o:o + L].view(1, L, hq, d), batch_offset=slots[b])
        o += L
    q_new = torch.full_like(q_ref, float("nan"))
    ops.gemm_qkv_rotary_varlen(x, w, lens, slots, hq, hk, d, cos, sin, c_new, q_new)
    assert ops.device_error() == 0
    torch.testing.assert_close(q_new.float(), q_ref.float(), rtol=2 ** -7, atol=1e-6)
    torch.testing.assert_close(c_new.float(), c_ref.float(), rtol=2 ** -7, atol=1e-6)
    unused = sorted(set(range(n + 1)) - set(slots))
    assert all(not c_new[u].any() for u in unused)
    # Slot n + 1 lies past the cache view's n + 1 rows: the guard row behind the view stays
    # untouched and the call reports a bad argument (its other outputs are then unspecified).
    guarded = torch.zeros(n + 2, cap, 2, hk, d, dtype=dt, device="cuda")
    ops.gemm_qkv_rotary_varlen(x, w, lens, [n + 1] + slots[1:], hq, hk, d, cos, sin,
                               guarded[:n + 1], torch.empty_like(q_ref))
    assert ops.device_error() == 2
    assert not guarded[n + 1].any()


@pytest.mark.parametrize("hq,hk,d", [(32, 32, 128), (32, 8, 128), (16, 2, 64)])
def test_prefill_attention_varlen_equals_per_prompt(ops, hq, hk, d):
    """Ragged prompts packed row after row (lengths 1, 127, 128, 129, 300, 700; permuted cache
    slots) in ONE varlen launch give exactly the per-prompt launches' outputs (same kernel work
    per query block) and match the FlashAttention-numerics oracle within 2e-2."""
    dt = torch.bfloat16
    lens = [129, 1, 700, 128, 127, 300]
    slots = [3, 0, 6, 1, 4, 2]
    B, cap = 7, 800
    g = torch.Generator().manual_seed(hq * 10 + d)
    cache_h = torch.randn(B, cap, 2, hk, d, generator=g).to(dt)
    q_h = torch.randn(sum(lens), hq, d, generator=g).to(dt)
    cache, q = cache_h.cuda(), q_h.cuda()
    scale = d ** -0.5
    out = torch.full_like(q, float("nan"))
    assert ops.prefill_attention_varlen(q, cache, lens, slots, hk, scale, out)
    zero = torch.zeros(1, dtype=torch.int32, device="cuda")
    o = 0
    for b, L in enumerate(lens):
        ref = ops.prefill_attention(q[o:o + L].view(1, L, hq, d), cache, zero, hk, scale,
                                    causal=True, batch_offset=slots[b])
        assert torch.equal(out[o:o + L], ref.view(L, hq, d)), b
        want = flash_attention(q_h[o:o + L][None], cache_h[slots[b], :L][None], True, scale)[0]
        torch.testing.assert_close(out[o:o + L].float().cpu(), want.float(), rtol=2e-2, atol=2e-2)
        o += L
    assert ops.device_error() == 0
    q32 = q.float()
    assert not ops.prefill_attention_varlen(q32, cache.float(), lens, slots, hk, scale,
                                            torch.empty_like(q32))
