/*
 * vjattn.h -- C ABI of the B200 (sm_100a) paged-attention hot path of
 * vllm-jax: KV-slot scatter fused with Qwen3 q/k RMSNorm + RoPE, split-KV
 * paged decode attention, varlen paged prefill attention, and the GPU
 * builder of the ragged batch metadata.
 *
 * Conventions shared by every entry point
 *   - All tensor arguments are DEVICE pointers owned by the caller (JAX
 *     buffers through an XLA FFI shim, torch tensors, or raw cudaMalloc).
 *     Dense activations are row-major bf16, indices are int32.
 *   - Nothing here allocates device memory. Kernels that need scratch take a
 *     caller-sized workspace whose size comes from a *_workspace_size query.
 *   - Every call is asynchronous on the given stream and never synchronises
 *     the host. Calls are reentrant; there is no hidden per-call state.
 *   - The return value is a vj_status. On a nonzero status nothing was
 *     launched and vj_get_last_error() returns a message for this thread.
 *   - KV pages are addressed by (block, token-in-block, kv-head, dim) with
 *     element strides, so both the engine's cache layout
 *     (2, num_blocks, block_size, Hkv, D) and the Pallas kernels' page
 *     layout (Hkv, num_blocks, page_size, D) are accepted without a copy.
 *
 * Reference interfaces replaced (paths inside the vllm-jax project):
 *   vj_kv_store_qknorm_rope   vllm/model/qwen3.py:105-111 (_update_kv_cache),
 *                             :59-78 (apply_rope), :286-296 (q/k norm+rope)
 *   vj_paged_decode           vllm/kernels/decode_paged_attention.py:300-397
 *                             (decode_paged_attention) incl. combine :274-283
 *   vj_paged_prefill          vllm/kernels/prefill_paged_attention.py:407-453
 *                             (prefill_paged_attention)
 *   vj_build_metadata         vllm/src/model_runner.py:204-301
 *                             (pad_block_tables, prepare_prefill, prepare_decode)
 */
#ifndef VJATTN_H_
#define VJATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef __CUDA_RUNTIME_H__
typedef struct CUstream_st *cudaStream_t;
#endif

#if defined(__GNUC__)
#define VJ_API __attribute__((visibility("default")))
#else
#define VJ_API
#endif

typedef int vj_status;
enum {
  VJ_OK = 0,
  VJ_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad shape, bad stride */
  VJ_ERR_UNSUPPORTED = 2,      /* valid but not implemented (e.g. head_dim != 128) */
  VJ_ERR_WORKSPACE = 3,        /* workspace missing or too small */
  VJ_ERR_CUDA = 4              /* a CUDA runtime/driver call failed */
};

/* Flags of vj_kv_store_qknorm_rope. */
enum {
  VJ_KV_NORM = 1,          /* apply per-head RMSNorm to q and k (weights required) */
  VJ_KV_ROPE = 2,          /* apply interleaved-pair RoPE to q and k */
  VJ_KV_WRAP_NEGATIVE = 4, /* slot s<0 writes slot s+num_slots, as JAX .at[] does */
  /* q_out = bf16(q / bf16(sqrt(D))): the reference's decode q scaling
   * (vllm/model/qwen3.py:207); attention then runs with scale 1 */
  VJ_KV_QSCALE_DIV_SQRT_D = 8,
  /* q_out = bf16(q * bf16(1/sqrt(D))): the reference's prefill kernel scaling
   * (vllm/kernels/prefill_paged_attention.py:60); attention then runs with scale 1 */
  VJ_KV_QSCALE_MUL_RSQRT_D = 16
};

/* Message of the last failed call on this host thread ("" if none). */
VJ_API const char *vj_get_last_error(void);

/* ABI version: (major << 16) | minor. */
VJ_API int vj_version(void);

/* ---------------------------------------------------------------------------
 * K3: q/k RMSNorm + RoPE + KV-slot scatter, one launch per layer.
 * Replaces vllm/model/qwen3.py:105-111 (_update_kv_cache, mode="drop") and
 * the q_norm/k_norm/apply_rope chain at qwen3.py:286-296 (apply_rope :59-78).
 *
 *   q_in [T,Hq,D], k_in [T,Hkv,D], v_in [T,Hkv,D] bf16; token t of each
 *   starts at base + t * *_row_stride elements (0 -> packed rows), so they
 *   may be column slices of one fused qkv projection output
 *   q_norm_w, k_norm_w [D] bf16 (required with VJ_KV_NORM)
 *   positions [T] int32, slot_mapping [T] int32 (flat slot = block*bs + offset)
 *   q_out [T,Hq,D] bf16 (may equal q_in), k_out [T,Hkv,D] bf16 or NULL
 *   k_cache/v_cache: element (blk,t,h,d) at base + blk*sb + t*st + h*sh + d
 *   rope_table [rope_table_len][D/2] (cos, sin) bf16 pairs from
 *   vj_rope_table_build for the same rope_theta; positions outside
 *   [0, rope_table_len) (or rope_table_len == 0) are computed in the kernel
 * Slots outside [0, num_blocks*block_size) are dropped (after the optional
 * negative wrap). Numerics: per row, squares summed in fp32 in a fixed order
 * (each of 8 lanes owning dims 8l..8l+7 and 64+8l..64+8l+7 sums its even and
 * its odd dims in dim order, adds the two, then a butterfly over lanes xor
 * 4, 2, 1);
 * every later step is a correctly rounded fp32 op followed by bf16
 * round-to-nearest-even, so the result is reproducible bit for bit.
 * ------------------------------------------------------------------------- */
VJ_API vj_status vj_kv_store_qknorm_rope(
    const void *q_in, const void *k_in, const void *v_in,
    const void *q_norm_w, const void *k_norm_w,
    const int32_t *positions, const int32_t *slot_mapping,
    void *q_out, void *k_out, void *k_cache, void *v_cache,
    int64_t num_tokens, int32_t num_q_heads, int32_t num_kv_heads,
    int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int64_t stride_block, int64_t stride_token, int64_t stride_head,
    int64_t q_row_stride, int64_t k_row_stride, int64_t v_row_stride,
    const void *rope_table, int32_t rope_table_len,
    float eps, float rope_theta, int32_t flags, cudaStream_t stream);

/* Number of bounded waits of vj_kv_store_qknorm_rope's staged kernel that
 * ran out (2 s each) since the library was loaded or last reset; nonzero means
 * a call's output is incomplete. Synchronous (reads a device word). No
 * counterpart in the reference. */
VJ_API vj_status vj_kv_store_timeouts(int32_t *count, int32_t reset);

/* RoPE table for vj_kv_store_qknorm_rope: for each position p < num_positions
 * and pair i < D/2, the bf16 word pair (cos, sin) of bf16(bf16(p) *
 * inv_freq[i]) (vllm/model/qwen3.py:62-67), inv_freq in bf16 from the bf16
 * rope_theta. Built once per model (positions repeat across layers and steps);
 * the caller allocates vj_rope_table_bytes() bytes, 16-byte aligned. */
VJ_API size_t vj_rope_table_bytes(int32_t num_positions, int32_t head_dim);
VJ_API vj_status vj_rope_table_build(void *table, int32_t num_positions, int32_t head_dim,
                                     float rope_theta, cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * K2: split-KV paged decode attention (one query token per sequence).
 * Replaces vllm/kernels/decode_paged_attention.py:300-397 together with its
 * XLA combine (:274-283) and the q scaling at vllm/model/qwen3.py:207.
 *
 *   q [B,Hq,D] bf16, out [B,Hq,D] bf16
 *   block_tables [B, bt_width] int32, row stride bt_stride (entries <0 are
 *   read as block 0, like the reference's safe_block_tables); a context
 *   longer than the table covers is truncated to bt_width*block_size tokens
 *   context_lens [B] int32 (0 -> out = 0)
 *   scale: softmax scale applied to q.k in fp32 (1/sqrt(D) for Qwen3)
 *   workspace: >= vj_paged_decode_workspace_size(B, Hq, D, max_chunks) bytes,
 *   16-byte aligned; max_chunks bounds the split count (0 -> default 4096).
 * ------------------------------------------------------------------------- */
VJ_API size_t vj_paged_decode_workspace_size(int32_t batch, int32_t num_q_heads,
                                      int32_t head_dim, int32_t max_chunks);

VJ_API vj_status vj_paged_decode(
    const void *q, const void *k_cache, const void *v_cache,
    const int32_t *block_tables, const int32_t *context_lens, void *out,
    int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
    int64_t num_blocks, int32_t block_size, int32_t bt_width, int32_t bt_stride,
    int64_t stride_block, int64_t stride_token, int64_t stride_head,
    float scale, int32_t max_chunks, void *workspace, size_t workspace_bytes,
    cudaStream_t stream);

/* vj_paged_decode without its planning launch: the workspace must hold the
 * plan of an earlier vj_paged_decode call on the same stream with the same
 * batch, context_lens values, num_kv_heads, bt_width, block_size and
 * max_chunks, with no call that used this workspace for another batch in
 * between. A decode step calls vj_paged_decode for its first layer and this
 * for the other layers (their lengths are the same). No counterpart in the
 * reference. */
VJ_API vj_status vj_paged_decode_planned(
    const void *q, const void *k_cache, const void *v_cache,
    const int32_t *block_tables, const int32_t *context_lens, void *out,
    int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
    int64_t num_blocks, int32_t block_size, int32_t bt_width, int32_t bt_stride,
    int64_t stride_block, int64_t stride_token, int64_t stride_head,
    float scale, int32_t max_chunks, void *workspace, size_t workspace_bytes,
    cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * K2 for callers that cannot allocate device memory. No counterpart in the
 * reference: it exists for callers such as a custom-call handler inside an
 * XLA/JAX computation (the runtime owns all device memory, and a cudaMalloc
 * there would bypass it and may synchronise the device) or a server that
 * fixes its memory budget at start-up.
 *
 * Same inputs, outputs and semantics as vj_paged_decode, without the
 * workspace: the split-KV scratch lives in a fixed 16 MiB device array
 * (vj_paged_decode_noalloc_scratch_bytes()) that every GPU loading this
 * library keeps until the process exits. Shapes whose scratch does not fit
 * (batch must stay below ~16 MiB / (Hq * 520 B), e.g. < 1008 sequences at
 * Hq = 32) return VJ_ERR_UNSUPPORTED. Its split budget (about 1008 - batch
 * chunks at Hq = 32, against 4096 + batch with a default workspace) allows
 * fewer splits, so batches of few long sequences run slower than through
 * vj_paged_decode. The first call in each CUDA context (each device, with
 * the runtime's primary contexts) looks up the array's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture. All calls on a device share the array and it
 * keeps the last call's contents (every word a call reads is rewritten by
 * that call first); calls whose kernels overlap on the GPU race on it, so
 * order them on one stream. It allocates nothing.
 * ------------------------------------------------------------------------- */
VJ_API size_t vj_paged_decode_noalloc_scratch_bytes(void);

VJ_API vj_status vj_paged_decode_noalloc(
    const void *q, const void *k_cache, const void *v_cache,
    const int32_t *block_tables, const int32_t *context_lens, void *out,
    int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
    int64_t num_blocks, int32_t block_size, int32_t bt_width, int32_t bt_stride,
    int64_t stride_block, int64_t stride_token, int64_t stride_head,
    float scale, cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * K1: varlen paged prefill attention (causal), tcgen05/TMEM tiles fed by TMA.
 * Replaces vllm/kernels/prefill_paged_attention.py:407-453
 * (prefill_paged_attention) incl. the Q gather (:227-239), split merge
 * (:364-376) and scatter to packed order (:384-388).
 *
 *   q [num_tokens, Hq, D] bf16 packed; sequence s owns rows
 *   [cu_seqlens_q[s], cu_seqlens_q[s+1]); out has the same shape, rows past
 *   cu_seqlens_q[num_seqs] are written as 0
 *   context_lens [num_seqs] int32 = cached prefix + new tokens (keys already
 *   in the pool), or NULL when keys == new tokens (the reference's case)
 *   new token i of sequence s sits at position context_len - n_s + i and
 *   attends to keys [0, that position]
 *   block_tables [num_seqs, bt_width] int32 (row stride bt_stride)
 *   max_seqlen_q: bound on new tokens per sequence (sizes the grid; <= 0 ->
 *   num_tokens), like the reference's static max_seqlen_bucket
 *   error_flag: device int32, set to 1 if a pipeline wait timed out
 * Query heads per KV head must divide 128; head_dim 128; block_size % 16 == 0.
 * ------------------------------------------------------------------------- */
VJ_API vj_status vj_paged_prefill(
    const void *q, const void *k_cache, const void *v_cache,
    const int32_t *block_tables, const int32_t *cu_seqlens_q,
    const int32_t *context_lens, void *out, int64_t num_tokens,
    int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads,
    int32_t head_dim, int64_t num_blocks, int32_t block_size, int32_t bt_width,
    int32_t bt_stride, int64_t stride_block, int64_t stride_token,
    int64_t stride_head, int32_t max_seqlen_q, float scale,
    int32_t *error_flag, cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * K1 + K2 in one launch for a chunked-prefill step that mixes decode rows
 * with prompt chunks (the reference schedules prefill and decode as separate
 * batches, vllm/src/scheduler.py:27-63, and has no such step; this replaces
 * the two attention calls such a step would make with one).
 *
 *   sequences [0, num_decode) are decode rows: q row b holds sequence b's one
 *   new token; sequences [num_decode, num_seqs) are prompt chunks after a
 *   cached prefix, rows [cu_seqlens_q[s], cu_seqlens_q[s+1]) as in
 *   vj_paged_prefill (cu_seqlens_q[s] == s for the decode rows); rows past
 *   cu_seqlens_q[num_seqs] (padding) are written as 0
 *   block_tables [num_seqs, bt_width], context_lens [num_seqs] (keys already
 *   in the pool, the new tokens included) for both kinds
 *   scale: applied to q.k in fp32 for both kinds
 *   workspace: decode split-KV scratch of
 *   vj_paged_attention_mixed_workspace_size(num_decode, Hq, D, max_chunks)
 *   bytes; plan = 0 reuses the split plan of an earlier call on the same
 *   stream with the same decode rows (the later layers of a step), as
 *   vj_paged_decode_planned does
 * Launches: the decode plan (plan != 0, decode rows present), one kernel
 * whose first CTAs run the split-KV decode warps, the next ones prefill tile
 * pairs and the last few zero the padding rows, and the decode combine.
 * error_flag as vj_paged_prefill.
 * ------------------------------------------------------------------------- */
VJ_API size_t vj_paged_attention_mixed_workspace_size(int32_t num_decode, int32_t num_q_heads,
                                                      int32_t head_dim, int32_t max_chunks);

VJ_API vj_status vj_paged_attention_mixed(
    const void *q, const void *k_cache, const void *v_cache,
    const int32_t *block_tables, const int32_t *cu_seqlens_q,
    const int32_t *context_lens, void *out, int64_t num_tokens, int32_t num_seqs,
    int32_t num_decode, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
    int64_t num_blocks, int32_t block_size, int32_t bt_width, int32_t bt_stride,
    int64_t stride_block, int64_t stride_token, int64_t stride_head, int32_t max_seqlen_q,
    float scale, int32_t max_chunks, int32_t plan, void *workspace, size_t workspace_bytes,
    int32_t *error_flag, cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * Fused decoder-layer epilogues (vllm/model/qwen3.py:375-389, :337-341).
 * vj_add_rmsnorm: r = bf16(x + residual) (stored to residual_out when given;
 * residual may be NULL for a plain norm), y = bf16(r * (rsqrt(mean(r^2) +
 * eps) * weight)) with fp32 statistics; rows x hidden bf16, hidden % 8 == 0,
 * hidden <= 8192. vj_silu_mul: out[t, i] = bf16(bf16(silu(g)) * u) for
 * gate_up = [g | u] of shape [rows, 2 * inter].
 * ------------------------------------------------------------------------- */
VJ_API vj_status vj_add_rmsnorm(const void *x, const void *residual,
                                const void *weight, void *residual_out, void *y,
                                int64_t rows, int32_t hidden, float eps,
                                cudaStream_t stream);
VJ_API vj_status vj_silu_mul(const void *gate_up, void *out, int64_t rows,
                             int32_t inter, cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * Decode-step projections (tcgen05 GEMM, bf16 in, fp32 accumulate) with the
 * next elementwise step fused into the epilogue. Built for decode batches
 * (rows up to a few hundred; at most 65536): every weight byte is read once,
 * the K dimension is split across CTAs as needed to fill the SMs, and split
 * partials are summed in a fixed order (results do not depend on timing).
 *
 * vj_decode_gemm, w [n, k] bf16 row-major (an nn.Linear weight), x [rows, k]
 * with row stride x_row_stride (0 -> k):
 *   VJ_GEMM_PLAIN   out[rows, n] = bf16(x w^T)
 *   VJ_GEMM_SWIGLU  w = [gate; up] (n = 2 I rows, I % 64 == 0):
 *                   out[rows, I] = bf16(bf16(silu(bf16(x gate^T))) * bf16(x up^T)),
 *                   the gate_up projection and vj_silu_mul in one launch
 *                   (vllm/model/qwen3.py:337-341)
 * vj_qkv_gemm_kv_store: the qkv projection (w_qkv = [Wq; Wk; Wv], rows
 *   (Hq + 2 Hkv) * 128, k = hidden) followed in the epilogue by exactly
 *   vj_kv_store_qknorm_rope's arithmetic on the bf16-rounded projections:
 *   q/k RMSNorm, RoPE, q scaling, q written to q_out [rows, Hq, 128] and k/v
 *   to their cache slots (qwen3.py:286-296, :105-111). Same flags and slot
 *   rules as vj_kv_store_qknorm_rope; k_out is not produced.
 * n and k: multiples of 128 and 64. splits: K split per output tile (0 ->
 * chosen from the shape and the SM count; at most 32). workspace: at least
 * vj_decode_gemm_workspace_size(rows, n, k, mode, splits) bytes (n = (Hq +
 * 2 Hkv) * 128 and VJ_GEMM_PLAIN for the qkv call), 256-byte aligned and
 * zero-filled once when allocated. Its first 64 KB hold the split tickets
 * (one word per output tile, whatever the shape), the fp32 split partials
 * follow, so one workspace serves calls of any shapes in stream order; calls
 * leave the tickets at zero unless error_flag (device int32, may be NULL) was
 * set, after which the workspace must be zero-filled again. A wait that runs
 * out (2 s) sets *error_flag = 1 and the call's outputs are incomplete.
 * ------------------------------------------------------------------------- */
enum { VJ_GEMM_PLAIN = 0, VJ_GEMM_SWIGLU = 1 };
/* weight_layout: VJ_WEIGHTS_ROW_MAJOR (w as given, read through a TMA tensor
 * map) or VJ_WEIGHTS_TILED (w packed once by vj_pack_weight_tiles with the
 * same n, k and mode; every pipeline stage is then one contiguous 16 KB bulk
 * copy, the faster weight stream). Both give bit-identical results. */
enum { VJ_WEIGHTS_ROW_MAJOR = 0, VJ_WEIGHTS_TILED = 1 };

VJ_API size_t vj_decode_gemm_workspace_size(int64_t rows, int32_t n, int32_t k, int32_t mode,
                                            int32_t splits);
/* Pack w [n, k] (mode VJ_GEMM_PLAIN, or VJ_GEMM_SWIGLU for [gate; up]) into
 * out (n * k bf16, distinct from w): 16 KB blocks of 128 weight rows x 64 K
 * in shared-memory swizzle order. */
VJ_API vj_status vj_pack_weight_tiles(const void *w, void *out, int32_t n, int32_t k,
                                      int32_t mode, cudaStream_t stream);
VJ_API vj_status vj_decode_gemm(const void *x, int64_t x_row_stride, const void *w,
                                int32_t weight_layout, void *out, int64_t out_row_stride,
                                int64_t rows, int32_t n, int32_t k, int32_t mode, int32_t splits,
                                void *workspace, size_t workspace_bytes, int32_t *error_flag,
                                cudaStream_t stream);
VJ_API vj_status vj_qkv_gemm_kv_store(
    const void *x, int64_t x_row_stride, const void *w_qkv, int32_t weight_layout,
    const void *q_norm_w,
    const void *k_norm_w, const int32_t *positions, const int32_t *slot_mapping, void *q_out,
    void *k_cache, void *v_cache, int64_t num_tokens, int32_t hidden, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int64_t stride_block, int64_t stride_token, int64_t stride_head, const void *rope_table,
    int32_t rope_table_len, float eps, float rope_theta, int32_t flags, int32_t splits,
    void *workspace, size_t workspace_bytes, int32_t *error_flag, cudaStream_t stream);

/* ---------------------------------------------------------------------------
 * K4: batch metadata built on the GPU from device-resident engine state.
 * Replaces vllm/src/model_runner.py:204-214 (pad_block_tables), :217-266
 * (prepare_prefill) and :268-301 (prepare_decode); the outputs equal the
 * reference's arrays element for element.
 *
 * Engine state, indexed by request slot (device, int32):
 *   token_table [max_slots, token_stride]  token ids of each request
 *   block_pool  [max_slots, bt_stride]     its allocated block ids
 *   num_blocks  [max_slots]                number of valid entries
 * Per call: seq_slots[num_seqs], seq_lens[num_seqs] (= len(request), or the
 * number of new tokens in VJ_META_RANGES mode), seq_starts[num_seqs] (ranges
 * mode only, else NULL: first new position, i.e. tokens already cached).
 * Prefill (mode VJ_META_PREFILL): all len tokens of each sequence, packed;
 *   input_ids/positions/slot_mapping [bucket_tokens] padded with 0/0/-1;
 *   cu_seqlens [bucket_batch + 1] padded by repeating the total;
 *   block_tables [bucket_batch, width] padded with -1.
 * Decode (VJ_META_DECODE): one row per sequence (last token, position
 *   len-1, context_lens = len), rows [num_seqs, bucket_tokens) padded with
 *   0/0/0/-1; block_tables [bucket_batch = bucket_tokens, width].
 *   flags & VJ_META_LAST_BLOCK_SLOT: slot = last allocated block * bs +
 *   (len-1) % bs, exactly as model_runner.py:282-284 (differs from the
 *   block holding position len-1 right after a block-boundary allocation).
 * error_flag (device int32) is set to 1 (position without an allocated
 * block), 2 (tokens exceed bucket_tokens) or 3 (bad scatter row).
 * ------------------------------------------------------------------------- */
enum { VJ_META_PREFILL = 0, VJ_META_DECODE = 1, VJ_META_RANGES = 2 };
enum { VJ_META_LAST_BLOCK_SLOT = 1 };

VJ_API vj_status vj_build_metadata(
    int32_t mode, const int32_t *seq_slots, const int32_t *seq_starts,
    const int32_t *seq_lens, int32_t num_seqs, const int32_t *token_table, int32_t token_stride,
    const int32_t *block_pool, const int32_t *num_blocks, int32_t bt_stride,
    int32_t block_size, int32_t width, int32_t bucket_tokens,
    int32_t bucket_batch, int32_t flags, int32_t *input_ids, int32_t *positions,
    int32_t *slot_mapping, int32_t *block_tables, int32_t *cu_seqlens,
    int32_t *context_lens, int32_t *error_flag, cudaStream_t stream);

/* Host-delta upload into a device table (block_pool or token_table):
 * headers [num_rows, 4] = (row, start, count, payload offset); writes
 * table[row][start, start+count) from payload and, if row_len is not NULL,
 * row_len[row] = start + count. A row may appear at most once per call. */
VJ_API vj_status vj_scatter_rows(const int32_t *headers, const int32_t *payload,
                                 int32_t num_rows, int32_t *table,
                                 int32_t table_stride, int32_t max_cols,
                                 int32_t *row_len, int32_t *error_flag,
                                 cudaStream_t stream);

/* Greedy sampling, vllm/sampler.py:13-15 (argmax over bf16 logits, first
 * index on ties): out_tokens[r] = argmax(logits[r, :vocab]); if token_table
 * is given the token is also stored at token_table[seq_slots[r]][seq_lens[r]]. */
VJ_API vj_status vj_argmax_append(const void *logits, int64_t row_stride,
                                  int32_t num_rows, int32_t vocab,
                                  int32_t *out_tokens, int32_t *token_table,
                                  int32_t token_stride, const int32_t *seq_slots,
                                  const int32_t *seq_lens, cudaStream_t stream);

/* Sampling, vllm/sampler.py:7-42 (the reference samples one request at a
 * time with one device->host copy each; this is one launch per batch).
 * Per row r: temperature[r] <= 0 -> argmax of the raw logits (first index on
 * ties). Otherwise x = bf16(logit / temperature[r]); top_k[r] > 0 keeps the
 * top_k largest x (equal values: lower index first); top_p[r] < 1 then keeps,
 * in (x desc, index asc) order, the tokens whose cumulative softmax
 * probability over the kept set is <= top_p[r] (the first always kept); the
 * token is drawn from softmax(x) over the kept set by Gumbel-max with
 * Philox4x32-10 keyed by seeds[2r], seeds[2r+1] and counter (vocab index,
 * seq_lens[r] or 0). num_kept (optional) receives the kept-set size.
 * token_table as in vj_argmax_append. logits must be 16-byte aligned with a
 * row stride that is a multiple of 8 elements. */
VJ_API vj_status vj_sample(const void *logits, int64_t row_stride, int32_t num_rows,
                           int32_t vocab, const float *temperature, const int32_t *top_k,
                           const float *top_p, const uint32_t *seeds,
                           int32_t *out_tokens, int32_t *num_kept, int32_t *token_table,
                           int32_t token_stride, const int32_t *seq_slots,
                           const int32_t *seq_lens, cudaStream_t stream);

/* ---- tensor parallelism over NVLink peer memory (no counterpart in the
 * reference, which runs on one device; its layer dataflow
 * vllm/model/qwen3.py:375-389 is what the fused op computes) ---- */
#define VJ_TP_MAX_RANKS 8
#define VJ_IPC_HANDLE_BYTES 64

/* Grid of vj_allreduce_add_rmsnorm on this device (4 CTAs per SM); every rank must
 * report the same value. */
VJ_API int32_t vj_tp_grid(void);
/* Bytes of the flag region at the start of a rank's communication memory:
 * flags [2][world][grid] u32, epochs [grid] u32, one error word. */
VJ_API size_t vj_tp_flags_bytes(int32_t world);
/* cudaMalloc'd, zeroed device memory that can be shared with
 * vj_ipc_get_handle (a torch caching-allocator block cannot). */
VJ_API vj_status vj_comm_alloc(size_t bytes, void **ptr);
VJ_API vj_status vj_comm_free(void *ptr);
/* cudaIpc handle (VJ_IPC_HANDLE_BYTES bytes) of a vj_comm_alloc pointer, and
 * its mapping in another process (peer access enabled lazily). */
VJ_API vj_status vj_ipc_get_handle(void *ptr, void *handle_out);
VJ_API vj_status vj_ipc_open_handle(const void *handle, void **ptr);
VJ_API vj_status vj_ipc_close_handle(void *ptr);

/* out = residual + sum over ranks of bufs[r][rows, hidden] (fp32 sum in rank
 * order, rounded to bf16, added in bf16) -> residual_out; y = RMSNorm(out) *
 * weight as vj_add_rmsnorm. bufs[r] is rank r's partial (peer pointers, own
 * included); peer_flags[r] the flag region of rank r; flags this rank's own.
 * results == NULL: one-shot (every rank reads every partial). Otherwise
 * results[r] is rank r's result buffer ([rows, hidden], peer pointers) and the
 * reduction is two-shot (reduce a slice, then gather the slices). Each CTA
 * signals its counterpart on every peer and waits for theirs (bounded: 2 s;
 * on timeout the error word of `flags` is set and the CTA returns). All ranks
 * must make the same sequence of calls; a buffer may be rewritten only after
 * the next call has been made by every rank (use two sets in alternation).
 * residual may be NULL (out = the sum). */
VJ_API vj_status vj_allreduce_add_rmsnorm(
    const void *const *bufs, void *const *results, uint32_t *const *peer_flags,
    uint32_t *flags, int32_t rank, int32_t world, const void *residual, const void *weight,
    void *residual_out, void *y, int64_t rows, int32_t hidden, float eps, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* VJATTN_H_ */
