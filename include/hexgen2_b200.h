/*
 * hexgen2_b200 — C ABI of the B200 (sm_100a) kernels behind the HexGen-2 prefill/decode path.
 *
 * Conventions shared by every entry point:
 *   - pointers are device pointers unless the name says "host";
 *   - sizes and strides are int64 element counts unless the name says "bytes";
 *   - `dtype` is an hx_dtype; `stream` is a cudaStream_t passed as void*;
 *   - the return value is an hx_status; on failure hx_last_error() describes it;
 *   - no entry point allocates device memory unless its comment says so: scratch space is
 *     passed in by the caller (size from the matching *_workspace() query).
 *
 * Reference interfaces replaced (paths are inside the HexGen-2 project):
 *   hexgen/hexgen_core/modules/rms_norm.py:13-15, modules/block.py:125-158 and
 *   models/gpt.py:388-397 (residual add + TorchRMSNorm), modules/embedding.py:37-51 and
 *   :111-124 (token embedding), modules/mha.py:255-288 and flash_attn RotaryEmbedding used at
 *   mha.py:557 (rotary + KV-cache write), nn.Linear at mha.py:395/:412, mlp.py:73-87 and
 *   models/gpt.py:440/:476 (projections), flash_attn_kvpacked_func at mha.py:141 (prefill and
 *   decode attention), hexgen2/model.py:81 and :103-109 (live KV slice / re-expansion),
 *   hexgen2/transport.py:44-80 (packet transfer of the KV cache), hexgen2/model.py:82/:117
 *   (greedy argmax).
 */
#ifndef HEXGEN2_B200_H
#define HEXGEN2_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum hx_dtype { HX_F32 = 0, HX_F16 = 1, HX_BF16 = 2 } hx_dtype;

typedef enum hx_status {
  HX_OK = 0,
  HX_ERR_INVALID = 1,     /* bad argument (shape, stride, alignment, null pointer) */
  HX_ERR_UNSUPPORTED = 2, /* valid request this build does not implement */
  HX_ERR_CUDA = 3,        /* a CUDA runtime call failed */
  HX_ERR_DEVICE = 4       /* a kernel reported a device-side error (see hx_device_error) */
} hx_status;

typedef enum hx_epilogue {
  HX_EPI_NONE = 0,     /* C = round(A B^T) */
  HX_EPI_RESIDUAL = 1, /* C = round(round(A B^T) + R)   (out_proj / fc2 + residual add) */
  HX_EPI_SWIGLU = 2,   /* B rows interleaved [up16|gate16]...; C[:, j] = up_j * silu(gate_j) */
  HX_EPI_QKV_ROTARY = 3 /* packed Wqkv output -> rotary q/k + KV-cache write (hx_gemm_qkv_rotary) */
} hx_epilogue;

/* ---------------------------------------------------------------- library / errors */
int hx_abi_version(void);
const char* hx_last_error(void);
/* Reads (and, if clear != 0, resets) the device-side error word that kernels set when a
 * bounded wait gives up. Synchronises the current device. */
int hx_device_error(int clear);
int hx_sm_count(void);

/* ---------------------------------------------------------------- embedding + norms */
/* out[r, :] = table[ids[r] - vocab_start, :] when vocab_start <= ids[r] < vocab_start+vocab_rows,
 * else zeros (vocab-parallel shard). Replaces GPT2Embeddings / VocabParallelEmbedding forward
 * (hexgen/hexgen_core/modules/embedding.py:37-51, :111-124). */
int hx_embedding(const int64_t* ids, int64_t rows, const void* table, int64_t vocab_start,
                 int64_t vocab_rows, int64_t hidden, void* out, int dtype, void* stream);

/* Fused embedding lookup + first-block RMSNorm (TP = 1):
 * residual_out[r] = table[ids[r]]; normed_out[r] = RMSNorm(residual_out[r]) * weight.
 * Replaces embedding.py:37-51 followed by block.py:126-129 for layer 0. */
int hx_embed_rmsnorm(const int64_t* ids, int64_t rows, const void* table, int64_t hidden,
                     const void* weight, float eps, void* residual_out, void* normed_out,
                     int dtype, void* stream);

/* Residual add + RMSNorm with the reference's rounding points:
 *   res = add ? round(x + add) : x;  residual_out (if non-null) = res;
 *   out = round(round(res * rsqrt(mean(res^2) + eps)) * weight)   (f32 statistics)
 * Row r of x/add is read at r*in_stride, outputs written at r*out_stride.
 * Replaces block.py:126-129 / :155-158 + rms_norm.py:13-15, and gpt.py:388-397 (ln_f). */
int hx_rmsnorm(const void* x, const void* add, void* residual_out, void* out,
               const void* weight, int64_t rows, int64_t hidden, int64_t in_stride,
               int64_t out_stride, float eps, int dtype, void* stream);

/* ---------------------------------------------------------------- rotary + cache write */
/* qkv: [batch, seqlen, (n_heads + 2*n_heads_kv) * head_dim] packed Wqkv output.
 * For token s of sequence b at position p = pos_start[b] + s (pos_start: device int32[batch]):
 *   q_out[b, s, h, :]              = rope(q[b, s, h, :], p)
 *   cache[cache_batch_offset + b, p, 0, hk, :] = rope(k[b, s, hk, :], p)
 *   cache[cache_batch_offset + b, p, 1, hk, :] = v[b, s, hk, :]
 * cos/sin tables are [table_rows, head_dim/2] in `dtype` (the reference caches them in the
 * activation dtype). interleaved != 0 rotates pairs (x[2i], x[2i+1]) (GPT-J style, what the
 * native Llama model uses); 0 rotates halves (GPT-NeoX style).
 * Replaces flash_attn RotaryEmbedding (mha.py:382-384, :557) + _update_kv_cache copy
 * (mha.py:255-288). */
int hx_rotary_cache_write(const void* qkv, int64_t batch, int64_t seqlen, int64_t n_heads,
                          int64_t n_heads_kv, int64_t head_dim, const int32_t* pos_start,
                          const void* cos_table, const void* sin_table, int64_t table_rows,
                          int interleaved, void* q_out, void* cache, int64_t cache_batch_stride,
                          int64_t cache_seq_stride, int64_t cache_batch_offset,
                          int64_t cache_max_seq, int dtype, void* stream);

/* ---------------------------------------------------------------- projections */
/* C[m, n] = A[m, k] * B[n, k]^T (both operands K-contiguous, nn.Linear weight layout), f32
 * accumulation, with the epilogue `epilogue` (hx_epilogue). f16/bf16 run on tcgen05 tensor
 * cores fed by TMA; f32 runs on a CUDA-core kernel (exact f32 products).
 * Alignment (f16/bf16): A, B 16-byte aligned; lda, ldb multiples of 8.
 * For HX_EPI_SWIGLU, n counts interleaved B rows (2 * intermediate) and C has n/2 columns.
 * `workspace` may be NULL when hx_gemm_workspace() returns 0 for the shape; otherwise it must
 * hold that many bytes (split-K partial sums).
 * Decode-shaped calls (m <= 64) use programmatic dependent launch and may start reading `b`
 * (the weight) before the previous kernel on the stream has finished, when that kernel is one of
 * this library's: `b` must not be written by the immediately preceding hx_* call on the stream
 * (weights never are). Every other input and the output wait for the previous kernel.
 * Replaces nn.Linear (mha.py:395/:412, mlp.py:73-87, gpt.py:440) + the residual add of
 * block.py:155-158 + the SwiGLU of mlp.py:79-87. */
int hx_gemm(const void* a, const void* b, void* c, int64_t m, int64_t n, int64_t k,
            int64_t lda, int64_t ldb, int64_t ldc, int epilogue, const void* residual,
            int64_t ld_residual, void* workspace, size_t workspace_bytes, int dtype,
            void* stream);
/* Workspace bytes for hx_gemm / hx_gemm_qkv_rotary: f32 split-K partial sums, needed only
 * when m > 64 and the output has too few tiles to fill the GPU (0 otherwise; decode-shaped
 * problems, m <= 64, reduce their K splits inside a thread-block cluster and never need one).
 * Calls that run concurrently need separate workspaces. */
size_t hx_gemm_workspace(int64_t m, int64_t n, int64_t k, int epilogue, int dtype);
/* Which kernel hx_gemm plans for a shape (host-only query, no GPU work): 0 CUDA-core f32,
 * 1 single-SM tcgen05 tiles (128 x 64..256, K split when the tiles are too few), 2 CTA-pair
 * tcgen05 tiles (256 x 256 over two SMs, cta_group::2), 3 decode-shaped (m <= 64: operands
 * swapped, K split inside a cluster). Diagnostic; no reference counterpart. */
int hx_gemm_kernel_kind(int64_t m, int64_t n, int64_t k, int dtype);

/* Wqkv projection fused with rotary and the KV-cache write: computes qkv = x * Wqkv^T
 * ([m, (n_heads + 2*n_heads_kv) * head_dim], f32 accumulation, rounded to dtype like the
 * reference's nn.Linear output) and, instead of storing it, writes exactly what
 * hx_rotary_cache_write would (interleaved rotary on q and k at position pos_start[b] + s for
 * row m = b * seqlen + s; q to q_out [m, n_heads, head_dim]; k, v to cache[cache_batch_offset
 * + b, pos]). f16/bf16 only. Replaces mha.py:542 + :557 + :286. */
int hx_gemm_qkv_rotary(const void* x, const void* w_qkv, int64_t m, int64_t k, int64_t ldx,
                       int64_t seqlen, int64_t n_heads, int64_t n_heads_kv, int64_t head_dim,
                       const int32_t* pos_start, const void* cos_table, const void* sin_table,
                       int64_t table_rows, void* q_out, void* cache, int64_t cache_batch_stride,
                       int64_t cache_seq_stride, int64_t cache_batch_offset,
                       int64_t cache_max_seq, void* workspace, size_t workspace_bytes, int dtype,
                       void* stream);

/* hx_gemm_qkv_rotary over prompts of different lengths packed row after row: prompt b owns
 * rows [seq_offsets[b], seq_offsets[b+1]) of x (n_prompts + 1 offsets, seq_offsets[0] = 0,
 * the last = m), and row seq_offsets[b] + s is rotated at position pos_start[b] + s and its k, v
 * go to cache[slots[b], pos] (0 <= slots[b] < cache_rows). seq_offsets, slots and pos_start are
 * device int32 arrays. A row whose slot or position falls outside the cache is never written and
 * sets the device error word to 2 (bad argument; see hx_device_error); the call's other outputs
 * are then unspecified, since waits that see the error word stop early. Replaces the per-prompt mha.py:542 + :557 + :286 of a
 * packed prefill pass in one launch. */
int hx_gemm_qkv_rotary_varlen(const void* x, const void* w_qkv, int64_t m, int64_t k,
                              int64_t ldx, const int32_t* seq_offsets, const int32_t* slots,
                              const int32_t* pos_start, int64_t n_prompts, int64_t n_heads,
                              int64_t n_heads_kv, int64_t head_dim, const void* cos_table,
                              const void* sin_table, int64_t table_rows, void* q_out, void* cache,
                              int64_t cache_batch_stride, int64_t cache_seq_stride,
                              int64_t cache_rows, int64_t cache_max_seq, void* workspace,
                              size_t workspace_bytes, int dtype, void* stream);

/* ---------------------------------------------------------------- attention */
/* Multi-query (prefill) attention over the KV cache written by hx_rotary_cache_write.
 * q: [batch, seqlen_q, n_heads, head_dim]; keys/values are cache[cache_batch_offset + b,
 * 0 : pos_start[b] + seqlen_q]. With causal != 0, query s of sequence b (position
 * pos_start[b] + s) attends to key positions <= pos_start[b] + s (FlashAttention's bottom-right
 * alignment); with causal == 0 every query attends to all of them (what the reference does
 * whenever sequence_len_offset > 0, mha.py:566-568). out: [batch, seqlen_q, n_heads, head_dim].
 * Replaces flash_attn_kvpacked_func(..., causal) at mha.py:141/:569. */
int hx_prefill_attention(const void* q, const void* cache, int64_t cache_batch_stride,
                         int64_t cache_seq_stride, int64_t cache_batch_offset,
                         const int32_t* pos_start, int64_t batch, int64_t seqlen_q,
                         int64_t n_heads, int64_t n_heads_kv, int64_t head_dim, int causal,
                         float softmax_scale, void* out, int dtype, void* stream);
/* Prefill attention of several prompts packed row after row in one launch (f16/bf16,
 * head_dim 64/128; HX_ERR_UNSUPPORTED otherwise, so the caller can attend prompt by prompt).
 * q/out: [total_rows, n_heads, head_dim]; prompt b owns rows [seq_offsets[b], seq_offsets[b+1])
 * and reads keys/values from cache row slots[b] (of cache_rows rows), positions
 * 0 : pos_start[b] + its length, with hx_prefill_attention's causal rule. items: n_items pairs
 * (prompt, 128-query block) of int32, every block of every prompt once, heaviest first for
 * causal work. All arrays live on the device. Same call site as hx_prefill_attention
 * (flash_attn_kvpacked_func, mha.py:141/:569), for the packed prefill of several requests. */
int hx_prefill_attention_varlen(const void* q, const void* cache, int64_t cache_batch_stride,
                                int64_t cache_seq_stride, int64_t cache_rows,
                                const int32_t* seq_offsets, const int32_t* slots,
                                const int32_t* pos_start, const int32_t* items, int64_t n_prompts,
                                int64_t n_items, int64_t total_rows, int64_t n_heads,
                                int64_t n_heads_kv, int64_t head_dim, int causal,
                                float softmax_scale, void* out, int dtype, void* stream);

/* Single-query decode attention, split over the key axis (flash-decoding), GQA aware.
 * q: [batch, n_heads, head_dim]; sequence b attends to cache[b, 0 : seqlens_k[b]]
 * (seqlens_k: device int32[batch], each <= max_seqlen_k). out: [batch, n_heads, head_dim].
 * workspace: hx_decode_attention_workspace() bytes of split partials.
 * Replaces flash_attn_kvpacked_func(..., causal=False) with q_len 1 at mha.py:565-569. */
int hx_decode_attention(const void* q, const void* cache, int64_t cache_batch_stride,
                        int64_t cache_seq_stride, const int32_t* seqlens_k, int64_t batch,
                        int64_t n_heads, int64_t n_heads_kv, int64_t head_dim,
                        int64_t max_seqlen_k, float softmax_scale, void* out, void* workspace,
                        size_t workspace_bytes, int dtype, void* stream);
size_t hx_decode_attention_workspace(int64_t batch, int64_t n_heads, int64_t head_dim,
                                     int64_t max_seqlen_k);

/* Scratch capacity of hx_decode_attention_noalloc (bytes, per GPU). */
#define HX_DECODE_NOALLOC_SCRATCH_BYTES (16u << 20)

/* hx_decode_attention for callers that cannot allocate device memory. This entry point has no
 * counterpart in the reference. Some callers of this library cannot call cudaMalloc: a host
 * runtime that owns a fixed device-memory budget and hands kernels only pre-carved buffers, a
 * process whose allocator belongs to another framework, or a latency-critical loop where an
 * allocation (which may synchronise the device) is not allowed. They pass the same inputs and
 * output as hx_decode_attention and no workspace: the split-KV partials go to a file-scope
 * device array of HX_DECODE_NOALLOC_SCRATCH_BYTES (16 MiB) that every GPU which loads the
 * library holds until the process exits. Shapes whose partials
 * (hx_decode_attention_workspace()) exceed that are rejected with HX_ERR_INVALID. The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress) with that device
 * current; make that first call before any CUDA-graph stream capture. All calls share the one
 * array and nothing in it needs to start at zero (every partial is written before it is read),
 * so calls that overlap on the GPU (different streams, concurrently) race with each other and
 * must be serialised by the caller. Allocates nothing. */
int hx_decode_attention_noalloc(const void* q, const void* cache, int64_t cache_batch_stride,
                                int64_t cache_seq_stride, const int32_t* seqlens_k,
                                int64_t batch, int64_t n_heads, int64_t n_heads_kv,
                                int64_t head_dim, int64_t max_seqlen_k, float softmax_scale,
                                void* out, int dtype, void* stream);

/* ---------------------------------------------------------------- sampling */
/* out_idx[r] = first index of the maximum of logits[r, 0:cols] (torch.argmax semantics).
 * Replaces logits.argmax(-1) at hexgen2/model.py:82 and :117. */
int hx_argmax(const void* logits, int64_t rows, int64_t cols, int64_t ld, int64_t* out_idx,
              int dtype, void* stream);

/* ---------------------------------------------------------------- KV handoff */
/* Gather-pack of live cache rows for n_req requests into one contiguous buffer.
 * Request r's source is viewed as [n_outer][cap_rows][row_bytes] starting at src_ptrs[r]
 * (outer stride outer_stride_bytes, row stride row_stride_bytes); its first live_rows[r]
 * rows of every outer slice are written densely to dst + dst_offsets[r] as
 * [n_outer][live_rows[r]][row_bytes]. src_ptrs/live_rows/dst_offsets are device arrays.
 * dst may be a peer GPU's buffer (peer access or IPC mapping): the copy then crosses NVLink
 * inside the kernel. Bytes are copied verbatim (row_bytes and all offsets multiples of 16).
 * Replaces the live slice t[:, :L].contiguous() at hexgen2/model.py:81 and the per-layer
 * sends of hexgen2/transport.py:54-59. */
int hx_kv_pack(const uint64_t* src_ptrs, const int64_t* live_rows, const int64_t* dst_offsets,
               int64_t n_req, int64_t n_outer, int64_t outer_stride_bytes,
               int64_t row_stride_bytes, int64_t row_bytes, int64_t max_live_rows, void* dst,
               void* stream);
/* Inverse of hx_kv_pack: scatter packed rows back into capacity-sized caches (dst_ptrs[r]).
 * Replaces the re-expansion into a full cache at hexgen2/model.py:103-109. */
int hx_kv_unpack(const void* src, const int64_t* src_offsets, const int64_t* live_rows,
                 const uint64_t* dst_ptrs, int64_t n_req, int64_t n_outer,
                 int64_t outer_stride_bytes, int64_t row_stride_bytes, int64_t row_bytes,
                 int64_t max_live_rows, void* stream);

/* Peer access / IPC plumbing for the NVLink handoff (one process per GPU). */
int hx_enable_peer_access(int peer_device);
int hx_ipc_get_handle(const void* device_ptr, void* handle_out_64_bytes);
int hx_ipc_open_handle(const void* handle_64_bytes, void** device_ptr_out);
int hx_ipc_close_handle(void* device_ptr);
/* Base address and size of the device allocation containing device_ptr (IPC handles refer to
 * whole allocations, so a sub-range is shared as handle + offset). */
int hx_mem_range(const void* device_ptr, void** base_out, size_t* size_out);
/* Copy-engine peer copy (cudaMemcpyPeerAsync) of `bytes` on `stream`. */
int hx_peer_copy(void* dst, int dst_device, const void* src, int src_device, size_t bytes,
                 void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HEXGEN2_B200_H */
