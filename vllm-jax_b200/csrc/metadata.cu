// K4: ragged batch metadata built on the GPU from device-resident engine state.
//
// Replaces the host loops of vllm/src/model_runner.py:204-301
// (pad_block_tables, prepare_prefill, prepare_decode) and their per-step
// H2D copies. The engine keeps, on the device and indexed by a request's
// "slot":
//   token_table [max_slots, token_stride]  every token id of the request
//   block_pool  [max_slots, bt_stride]     block ids allocated to the request
//   num_blocks  [max_slots]                how many of them are valid
// and uploads per step only the scheduled (slot, length) pairs plus the rows
// that changed (vj_scatter_rows). vj_argmax_append writes each sampled token
// straight into token_table, so a decode step's input ids never leave the GPU.
//
// Integer work only, HBM/latency bound (a few KB per step): the aim is to
// remove host loops and launches of copies, not FLOPs.
#include "../../include/vjattn.h"
#include "vj_common.cuh"

#include <string>

namespace vj {
namespace {

constexpr int kMetaThreads = 512;
constexpr int kMaxSeqsScan = 8192;   // sequences per step handled by the in-CTA scan

struct MetaArgs {
  int mode;  // VJ_META_PREFILL / VJ_META_DECODE / VJ_META_RANGES
  const int32_t *seq_slots, *seq_lens;
  const int32_t *seq_starts;  // VJ_META_RANGES: first new position of each sequence
  int num_seqs;
  const int32_t *token_table;
  int token_stride;
  const int32_t *block_pool, *num_blocks;
  int bt_stride, block_size, width, bucket_tokens, bucket_batch, flags;
  int32_t *input_ids, *positions, *slot_mapping, *block_tables, *cu_seqlens, *context_lens;
  int32_t *error_flag;
};

// Flat slot of position `pos` of a request (model_runner.py:232-236).
__device__ inline int32_t slot_of(const MetaArgs &a, int slot, int pos) {
  const int nblk = __ldg(a.num_blocks + slot);
  const int bi = pos / a.block_size;
  if (bi >= nblk) return -1;  // not allocated: reported through error_flag
  return __ldg(a.block_pool + (size_t)slot * a.bt_stride + bi) * a.block_size + pos % a.block_size;
}

__global__ void __launch_bounds__(kMetaThreads)
build_metadata_kernel(MetaArgs a) {
  __shared__ int32_t cu[kMaxSeqsScan + 1];
  __shared__ int32_t warp_sums[kMetaThreads / 32];
  const int tid = threadIdx.x;
  const int S = a.num_seqs;

  if (a.mode == VJ_META_PREFILL || a.mode == VJ_META_RANGES) {
    // ---- cu_seqlens: exclusive scan of the lengths (every CTA redoes it; S is small)
    const int per = (S + kMetaThreads - 1) / kMetaThreads;
    const int b0 = tid * per;
    int local = 0;
    for (int s = b0; s < b0 + per && s < S; ++s) local += __ldg(a.seq_lens + s);
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if ((tid & 31) >= o) incl += v;
    }
    if ((tid & 31) == 31) warp_sums[tid >> 5] = incl;
    __syncthreads();
    if (tid < 32) {
      int w = tid < kMetaThreads / 32 ? warp_sums[tid] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, w, o);
        if (tid >= o) w += v;
      }
      if (tid < kMetaThreads / 32) warp_sums[tid] = w;  // inclusive over warps
    }
    __syncthreads();
    int run = incl - local + ((tid >> 5) > 0 ? warp_sums[(tid >> 5) - 1] : 0);
    for (int s = b0; s < b0 + per && s < S; ++s) {
      cu[s] = run;
      run += __ldg(a.seq_lens + s);
    }
    if (tid == 0) cu[0] = 0;
    __syncthreads();
    const int total = S > 0 ? cu[S - 1] + __ldg(a.seq_lens + S - 1) : 0;
    if (tid == 0) cu[S] = total;
    __syncthreads();
    if (total > a.bucket_tokens && blockIdx.x == 0 && tid == 0) atomicExch(a.error_flag, 2);

    const int gtid = blockIdx.x * kMetaThreads + tid;
    const int gstride = gridDim.x * kMetaThreads;
    // ---- per-token ids, positions and slots; bucket padding (0, 0, -1)
    for (int t = gtid; t < a.bucket_tokens; t += gstride) {
      int32_t id = 0, pos = 0, sl = -1;
      if (t < total) {
        int lo = 0, hi = S - 1;  // last s with cu[s] <= t
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (cu[mid] <= t) lo = mid; else hi = mid - 1;
        }
        const int slot = __ldg(a.seq_slots + lo);
        pos = t - cu[lo] + (a.mode == VJ_META_RANGES ? __ldg(a.seq_starts + lo) : 0);
        id = __ldg(a.token_table + (size_t)slot * a.token_stride + pos);
        sl = slot_of(a, slot, pos);
        if (sl < 0) atomicExch(a.error_flag, 1);
      }
      a.input_ids[t] = id;
      a.positions[t] = pos;
      a.slot_mapping[t] = sl;
    }
    // ---- cu_seqlens padded to bucket_batch + 1 by repeating the total
    for (int s = gtid; s <= a.bucket_batch; s += gstride) {
      a.cu_seqlens[s] = s <= S ? cu[s] : total;
    }
    // ---- ranges: keys per sequence = start + new tokens (0 for padding rows)
    if (a.mode == VJ_META_RANGES && a.context_lens) {
      for (int s = gtid; s < a.bucket_batch; s += gstride) {
        a.context_lens[s] = s < S ? __ldg(a.seq_starts + s) + __ldg(a.seq_lens + s) : 0;
      }
    }
  } else {
    // ---- decode: one row per scheduled sequence, padding (0, 0, ctx 0, slot -1)
    const int gtid = blockIdx.x * kMetaThreads + tid;
    const int gstride = gridDim.x * kMetaThreads;
    for (int b = gtid; b < a.bucket_tokens; b += gstride) {
      int32_t id = 0, pos = 0, ctx = 0, sl = -1;
      if (b < S) {
        const int slot = __ldg(a.seq_slots + b);
        const int len = __ldg(a.seq_lens + b);
        pos = len - 1;
        ctx = len;
        id = __ldg(a.token_table + (size_t)slot * a.token_stride + pos);
        if (a.flags & VJ_META_LAST_BLOCK_SLOT) {
          // model_runner.py:282-284: the LAST allocated block, offset (len-1) % bs
          const int nblk = __ldg(a.num_blocks + slot);
          sl = nblk > 0 ? __ldg(a.block_pool + (size_t)slot * a.bt_stride + nblk - 1) *
                              a.block_size + pos % a.block_size
                        : -1;
        } else {
          sl = slot_of(a, slot, pos);
        }
        if (sl < 0) atomicExch(a.error_flag, 1);
      }
      a.input_ids[b] = id;
      a.positions[b] = pos;
      a.slot_mapping[b] = sl;
      if (a.context_lens) a.context_lens[b] = ctx;
    }
  }
  // ---- block tables [bucket_batch, width]: allocated blocks, then -1
  // (model_runner.py:204-214)
  const int gtid = blockIdx.x * kMetaThreads + tid;
  const int gstride = gridDim.x * kMetaThreads;
  const long long cells = (long long)a.bucket_batch * a.width;
  for (long long c = gtid; c < cells; c += gstride) {
    const int row = (int)(c / a.width), col = (int)(c % a.width);
    int32_t v = -1;
    if (row < S) {
      const int slot = __ldg(a.seq_slots + row);
      if (col < __ldg(a.num_blocks + slot)) v = __ldg(a.block_pool + (size_t)slot * a.bt_stride + col);
    }
    a.block_tables[c] = v;
  }
}

// Row scatter of host deltas into a device table: header i = (row, start,
// count, payload offset); writes table[row][start : start + count] and, when
// row_len is given, row_len[row] = start + count.
__global__ void scatter_rows_kernel(const int32_t *__restrict__ headers,
                                    const int32_t *__restrict__ payload, int num_rows,
                                    int32_t *table, int table_stride, int max_cols,
                                    int32_t *row_len, int32_t *error_flag) {
  const int i = blockIdx.x;
  if (i >= num_rows) return;
  const int row = __ldg(headers + 4 * i), start = __ldg(headers + 4 * i + 1);
  const int count = __ldg(headers + 4 * i + 2), off = __ldg(headers + 4 * i + 3);
  if (row < 0 || start < 0 || count < 0 || start + count > max_cols) {
    if (threadIdx.x == 0) atomicExch(error_flag, 3);
    return;
  }
  for (int c = threadIdx.x; c < count; c += blockDim.x) {
    table[(size_t)row * table_stride + start + c] = __ldg(payload + off + c);
  }
  if (row_len && threadIdx.x == 0) row_len[row] = start + count;
}

// Greedy sampling (vllm/sampler.py:13-15: argmax, first index on ties) of
// rows [0, num_rows) of bf16 logits, one CTA per row; the token is written to
// out_tokens[row] and appended to the request's token_table row at column
// seq_lens[row] when token_table is given.
__global__ void __launch_bounds__(1024)
argmax_append_kernel(const __nv_bfloat16 *__restrict__ logits, int64_t row_stride, int vocab,
                     int32_t *out_tokens, int32_t *token_table, int token_stride,
                     const int32_t *seq_slots, const int32_t *seq_lens) {
  const int row = blockIdx.x;
  const __nv_bfloat16 *x = logits + (size_t)row * row_stride;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
    float v = __bfloat162float(x[i]);
    if (v != v) v = INFINITY;  // NaN ranks first, as in jnp.argmax
    if (v > best || (v == best && i < idx)) { best = v; idx = i; }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
  }
  if ((threadIdx.x & 31) == 0) { sb[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = idx; }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    best = threadIdx.x < nw ? sb[threadIdx.x] : -INFINITY;
    idx = threadIdx.x < nw ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
    }
    if (threadIdx.x == 0) {
      if (idx == 0x7fffffff) idx = 0;
      out_tokens[row] = idx;
      if (token_table) {
        const int slot = seq_slots[row], len = seq_lens[row];
        if (len >= 0 && len < token_stride) token_table[(size_t)slot * token_stride + len] = idx;
      }
    }
  }
}

}  // namespace
}  // namespace vj

extern "C" vj_status vj_build_metadata(
    int32_t mode, const int32_t *seq_slots, const int32_t *seq_starts, const int32_t *seq_lens,
    int32_t num_seqs,
    const int32_t *token_table, int32_t token_stride, const int32_t *block_pool,
    const int32_t *num_blocks, int32_t bt_stride, int32_t block_size, int32_t width,
    int32_t bucket_tokens, int32_t bucket_batch, int32_t flags, int32_t *input_ids,
    int32_t *positions, int32_t *slot_mapping, int32_t *block_tables, int32_t *cu_seqlens,
    int32_t *context_lens, int32_t *error_flag, cudaStream_t stream) {
  using namespace vj;
  if (mode != VJ_META_PREFILL && mode != VJ_META_DECODE && mode != VJ_META_RANGES) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_build_metadata: mode must be prefill, decode or ranges");
  }
  if (mode == VJ_META_RANGES && !seq_starts) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_build_metadata: ranges need seq_starts");
  }
  if (num_seqs < 0 || token_stride <= 0 || bt_stride < width || block_size <= 0 || width < 0 ||
      bucket_tokens < 0 || bucket_batch < 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_build_metadata: negative or inconsistent size");
  }
  if (mode == VJ_META_DECODE && bucket_tokens < num_seqs) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_build_metadata: decode bucket smaller than batch");
  }
  if (mode != VJ_META_DECODE && (bucket_batch < num_seqs || num_seqs > kMaxSeqsScan)) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_build_metadata: prefill needs num_seqs <= bucket_batch and <= 8192");
  }
  if (!seq_slots || !seq_lens || !token_table || !block_pool || !num_blocks || !input_ids ||
      !positions || !slot_mapping || !block_tables || !error_flag ||
      (mode != VJ_META_DECODE && !cu_seqlens)) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_build_metadata: null pointer");
  }
  MetaArgs a;
  a.mode = mode; a.seq_slots = seq_slots; a.seq_starts = seq_starts; a.seq_lens = seq_lens;
  a.num_seqs = num_seqs;
  a.token_table = token_table; a.token_stride = token_stride;
  a.block_pool = block_pool; a.num_blocks = num_blocks;
  a.bt_stride = bt_stride; a.block_size = block_size; a.width = width;
  a.bucket_tokens = bucket_tokens; a.bucket_batch = bucket_batch; a.flags = flags;
  a.input_ids = input_ids; a.positions = positions; a.slot_mapping = slot_mapping;
  a.block_tables = block_tables; a.cu_seqlens = cu_seqlens; a.context_lens = context_lens;
  a.error_flag = error_flag;
  const long long work = (long long)bucket_tokens + (long long)bucket_batch * width;
  int grid = (int)((work + kMetaThreads * 4 - 1) / (kMetaThreads * 4));
  if (grid < 1) grid = 1;
  if (grid > num_sms() * 4) grid = num_sms() * 4;
  build_metadata_kernel<<<grid, kMetaThreads, 0, stream>>>(a);
  return check_launch("vj_build_metadata");
}

extern "C" vj_status vj_scatter_rows(const int32_t *headers, const int32_t *payload,
                                     int32_t num_rows, int32_t *table, int32_t table_stride,
                                     int32_t max_cols, int32_t *row_len, int32_t *error_flag,
                                     cudaStream_t stream) {
  using namespace vj;
  if (num_rows < 0 || table_stride < max_cols || max_cols < 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_scatter_rows: bad sizes");
  }
  if (num_rows == 0) return VJ_OK;
  if (!headers || !payload || !table || !error_flag) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_scatter_rows: null pointer");
  }
  scatter_rows_kernel<<<num_rows, 128, 0, stream>>>(headers, payload, num_rows, table,
                                                    table_stride, max_cols, row_len, error_flag);
  return check_launch("vj_scatter_rows");
}

extern "C" vj_status vj_argmax_append(const void *logits, int64_t row_stride, int32_t num_rows,
                                      int32_t vocab, int32_t *out_tokens, int32_t *token_table,
                                      int32_t token_stride, const int32_t *seq_slots,
                                      const int32_t *seq_lens, cudaStream_t stream) {
  using namespace vj;
  if (num_rows < 0 || vocab <= 0 || row_stride < vocab) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_argmax_append: bad sizes");
  }
  if (num_rows == 0) return VJ_OK;
  if (!logits || !out_tokens || (token_table && (!seq_slots || !seq_lens))) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_argmax_append: null pointer");
  }
  argmax_append_kernel<<<num_rows, 1024, 0, stream>>>(
      static_cast<const __nv_bfloat16 *>(logits), row_stride, vocab, out_tokens, token_table,
      token_stride, seq_slots, seq_lens);
  return check_launch("vj_argmax_append");
}
