// K2: split-KV paged decode attention (one query token per sequence, GQA).
//
// Replaces vllm/kernels/decode_paged_attention.py:300-397 (vmap over the
// batch of paged_attention_unbatched :152-283, kernel :34-147) and its XLA
// combine :274-283, plus the bf16 q scaling at vllm/model/qwen3.py:207.
//
// Three launches on the caller's stream:
//   1. decode_plan_kernel  (1 CTA): pages per sequence, chunk size from the
//      real lengths (the reference splits by table width instead), per-
//      sequence chunk offsets, and a reset of the dynamic work counter.
//   2. decode_chunk_kernel (persistent, 2 CTAs/SM x 4 warps): each warp pulls
//      work items (chunk, kv-head) from an atomic counter and streams the
//      chunk's 16-token K/V pages through a private TMA ring (3 x 8 KB). QK^T
//      and PV run on mma.sync m16n8k16 with the GQA group as the M rows, so
//      every K/V byte is read from HBM exactly once for all g query heads.
//      Online softmax in fp32 with exp2; the quad of lanes sharing a row
//      reduces with warp shuffles. A sequence that fits one chunk writes its
//      final bf16 output directly; otherwise the chunk writes fp32 partials.
//   3. decode_combine_kernel: log-sum-exp merge of the partials (fp32).
// HBM-bound: bytes = sum(ctx)*Hkv*D*2*2 + q/out + block tables.
#include "../../include/vjattn.h"
#include "vj_common.cuh"

#include <mutex>
#include <string>

namespace vj {
namespace {

constexpr int kD = 128;
constexpr int kPageTok = 16;                 // tokens per TMA page box
constexpr int kWarps = 4;                    // warps per CTA
constexpr int kStages = 3;                   // pages in flight per warp
constexpr int kHalfBytes = kPageTok * 128;   // 16 rows x 64 dims x bf16
constexpr int kStageBytes = 4 * kHalfBytes;  // K lo/hi + V lo/hi
constexpr int kCtasPerSm = 2;
constexpr int kMinChunkPages = 8;
constexpr int kItemsPerWarp = 8;
constexpr float kLog2e = 1.4426950408889634f;

struct Workspace {
  int32_t *meta;     // [0]=pages/chunk, [1]=total chunks, [2]=item counter
  int32_t *prefix;   // [B+1] first chunk of each sequence
  float2 *part_ml;   // [max_chunks, Hq] (m in log2 units, l)
  float *part_o;     // [max_chunks, Hq, D]
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline Workspace carve(void *base, int B, int Hq, int max_chunks) {
  Workspace w;
  char *p = static_cast<char *>(base);
  w.meta = reinterpret_cast<int32_t *>(p);
  size_t off = 64;
  w.prefix = reinterpret_cast<int32_t *>(p + off);
  off = align_up(off + sizeof(int32_t) * (B + 1), 256);
  w.part_ml = reinterpret_cast<float2 *>(p + off);
  off = align_up(off + sizeof(float2) * (size_t)max_chunks * Hq, 256);
  w.part_o = reinterpret_cast<float *>(p + off);
  return w;
}

inline size_t workspace_bytes(int B, int Hq, int max_chunks) {
  size_t off = 64;
  off = align_up(off + sizeof(int32_t) * (B + 1), 256);
  off = align_up(off + sizeof(float2) * (size_t)max_chunks * Hq, 256);
  off += sizeof(float) * (size_t)max_chunks * Hq * kD;
  return align_up(off, 256);
}

// Pages (16-token boxes) of a sequence, capped by the block-table width.
__device__ inline int pages_of(int len, int max_pages) {
  const int p = len > 0 ? (len + kPageTok - 1) / kPageTok : 0;
  return p < max_pages ? p : max_pages;
}

// One CTA of 1024 threads. Chunk size: enough chunks for ~kItemsPerWarp items
// per resident warp, never more than max_chunks in total, never below
// kMinChunkPages pages.
__global__ void __launch_bounds__(1024)
decode_plan_kernel(const int32_t *__restrict__ lens, int B, int Hkv, int max_chunks,
                   int total_warps, int max_pages, Workspace ws) {
  __shared__ long long red[32];
  __shared__ int scan[1024];
  const int tid = threadIdx.x;
  long long mine = 0;
  for (int b = tid; b < B; b += 1024) mine += pages_of(lens[b], max_pages);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
  if ((tid & 31) == 0) red[tid >> 5] = mine;
  __syncthreads();
  if (tid < 32) {
    long long v = red[tid];
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    red[tid] = v;  // every lane holds the total
  }
  __syncthreads();
  const long long total_pages = red[0];
  long long cap = (long long)max_chunks - B;
  long long want = (long long)kItemsPerWarp * total_warps / (Hkv > 0 ? Hkv : 1);
  if (want < 1) want = 1;
  long long target = want < cap ? want : cap;
  if (target < 1) target = 1;
  long long P = (total_pages + target - 1) / target;
  if (P < kMinChunkPages) P = kMinChunkPages;

  // exclusive scan of chunks per sequence; thread tid owns a contiguous run
  const int per = (B + 1023) / 1024;
  const int b0 = tid * per;
  int local = 0;
  for (int b = b0; b < b0 + per && b < B; ++b) {
    local += (int)((pages_of(lens[b], max_pages) + P - 1) / P);
  }
  scan[tid] = local;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    int v = tid >= o ? scan[tid - o] : 0;
    __syncthreads();
    scan[tid] += v;
    __syncthreads();
  }
  int run = scan[tid] - local;
  for (int b = b0; b < b0 + per && b < B; ++b) {
    ws.prefix[b] = run;
    run += (int)((pages_of(lens[b], max_pages) + P - 1) / P);
  }
  if (tid == 1023) {
    ws.prefix[B] = scan[1023];
    ws.meta[0] = (int)P;
    ws.meta[1] = scan[1023];
    ws.meta[2] = 0;
    ws.meta[3] = 0;
  }
}

struct DecodeArgs {
  const __nv_bfloat16 *q;
  __nv_bfloat16 *out;
  const int32_t *bt;
  const int32_t *lens;
  int B, Hq, Hkv, g, bt_stride, pages_per_block, block_size;
  int max_pages;   // bt_width * pages_per_block
  int num_blocks;
  int head_major;  // 1: tensor map dims are (D, Hkv, tokens); 0: (D, tokens, Hkv)
  float scale_log2;
  Workspace ws;
};

struct Cursor {
  int item;    // work item id, or -1 when the queue is drained
  int b, h;    // sequence, kv head
  int chunk;   // global chunk id
  int p;       // next page (sequence-relative)
  int p_end;   // one past the last page of the chunk
};

__device__ inline int upper_bound_prefix(const int32_t *prefix, int B, int x) {
  int lo = 0, hi = B;  // find last b with prefix[b] <= x
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (__ldg(prefix + mid) <= x) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ inline void cursor_next_item(Cursor &c, const DecodeArgs &a, int total_items,
                                        int lane) {
  int it = 0;
  if (lane == 0) it = atomicAdd(a.ws.meta + 2, 1);
  it = __shfl_sync(0xffffffffu, it, 0);
  if (it >= total_items) { c.item = -1; return; }
  c.item = it;
  c.chunk = it / a.Hkv;
  c.h = it % a.Hkv;
  c.b = upper_bound_prefix(a.ws.prefix, a.B, c.chunk);
  const int P = a.ws.meta[0];
  const int k = c.chunk - __ldg(a.ws.prefix + c.b);
  const int np = pages_of(__ldg(a.lens + c.b), a.max_pages);
  c.p = k * P;
  c.p_end = min(np, c.p + P);
}

__global__ void __launch_bounds__(kWarps * 32, kCtasPerSm)
decode_chunk_kernel(const __grid_constant__ CUtensorMap tmk,
                    const __grid_constant__ CUtensorMap tmv, DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t *ring = smem + warp * (kStages * kStageBytes);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kWarps * kStages * kStageBytes) +
                   warp * kStages;
  // per stage: item id of the page it holds (-1 = drained), page index
  int *st_item = reinterpret_cast<int *>(full + (kWarps - warp) * kStages) +
                 warp * kStages * 4;

  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    if (warp == 0) { tma_prefetch_desc(&tmk); tma_prefetch_desc(&tmv); }
  }
  __syncwarp();

  const int total_items = a.ws.meta[1] * a.Hkv;
  Cursor pc;  // producer cursor (runs kStages pages ahead)
  pc.item = 0; pc.p = 0; pc.p_end = 0;

  // issue the next page of the producer cursor into stage s
  auto produce = [&](int s) {
    while (pc.item >= 0 && pc.p >= pc.p_end) cursor_next_item(pc, a, total_items, lane);
    if (lane == 0) {
      int *info = st_item + s * 4;
      if (pc.item < 0) {
        info[0] = -1;
        mbar_arrive(&full[s]);
      } else {
        const int page = pc.p;
        int blk = __ldg(a.bt + (size_t)pc.b * a.bt_stride + page / a.pages_per_block);
        if (blk < 0 || blk >= a.num_blocks) blk = 0;  // safe_block_tables
        const int tok0 = blk * a.block_size + (page % a.pages_per_block) * kPageTok;
        info[0] = pc.item; info[1] = page; info[2] = pc.b; info[3] = pc.h | (pc.chunk << 8);
        uint8_t *dst = ring + s * kStageBytes;
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        const int c1 = a.head_major ? pc.h : tok0, c2 = a.head_major ? tok0 : pc.h;
        tma_load_3d(dst, &tmk, &full[s], 0, c1, c2);
        tma_load_3d(dst + kHalfBytes, &tmk, &full[s], 64, c1, c2);
        tma_load_3d(dst + 2 * kHalfBytes, &tmv, &full[s], 0, c1, c2);
        tma_load_3d(dst + 3 * kHalfBytes, &tmv, &full[s], 64, c1, c2);
      }
    }
    if (pc.item >= 0) pc.p++;
  };

  for (int s = 0; s < kStages; ++s) produce(s);

  const int r = lane >> 2, qd = lane & 3;
  uint32_t qa0[8], qa2[8];
  float acc[16][4];
  float m_run = -INFINITY, l_run = 0.f;
  int cur_item = -1, len = 0, b = 0, h = 0, chunk = 0, page_end = 0;
  bool fail = false;

  for (int it = 0;; ++it) {
    const int s = it % kStages;
    const uint32_t parity = (it / kStages) & 1;
    if (!mbar_wait(&full[s], parity)) { fail = true; break; }
    const int *info = st_item + s * 4;
    const int item = info[0];
    if (item < 0) break;
    const int page = info[1];

    if (item != cur_item) {
      cur_item = item;
      b = info[2]; h = info[3] & 0xff; chunk = info[3] >> 8;
      len = __ldg(a.lens + b);
      const int P = a.ws.meta[0];
      const int np = pages_of(len, a.max_pages);
      page_end = min(np, (chunk - __ldg(a.ws.prefix + b)) * P + P);
      m_run = -INFINITY; l_run = 0.f;
#pragma unroll
      for (int n = 0; n < 16; ++n) { acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f; }
      if (r < a.g) {
        const uint32_t *qrow = reinterpret_cast<const uint32_t *>(
            a.q + ((size_t)b * a.Hq + (size_t)h * a.g + r) * kD);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          qa0[ks] = __ldg(qrow + ks * 8 + qd);
          qa2[ks] = __ldg(qrow + ks * 8 + 4 + qd);
        }
      } else {
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) { qa0[ks] = 0u; qa2[ks] = 0u; }
      }
    }

    const uint32_t kb = smem_u32(ring + s * kStageBytes);
    const uint32_t vb = kb + 2 * kHalfBytes;
    // ---- S = Q K^T over the page's 16 tokens (2 n-tiles of 8)
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
      const uint32_t row = (lane & 7) + ((lane >> 4) << 3);
      const uint32_t csel = (lane >> 3) & 1;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t half = ks >> 2;
        const uint32_t chunk16 = ((ks & 3) << 1) + csel;
        uint32_t b00, b01, b10, b11;
        ldsm_x4(kb + half * kHalfBytes + sw128(row, chunk16), b00, b01, b10, b11);
        mma_bf16_16816(sc[0], qa0[ks], 0u, qa2[ks], 0u, b00, b01);
        mma_bf16_16816(sc[1], qa0[ks], 0u, qa2[ks], 0u, b10, b11);
      }
    }
    // ---- online softmax (rows r = query heads; quad lanes share a row)
    float mx = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int tok = page * kPageTok + nt * 8 + qd * 2 + j;
        const float v = tok < len ? sc[nt][j] * a.scale_log2 : -INFINITY;
        sc[nt][j] = v;
        mx = fmaxf(mx, v);
      }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float m_use = m_new == -INFINITY ? 0.f : m_new;
    const float corr = fast_exp2(m_run - m_use);
    m_run = m_new;
    float ps = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        sc[nt][j] = fast_exp2(sc[nt][j] - m_use);
        ps += sc[nt][j];
      }
    }
    l_run = l_run * corr + ps;
#pragma unroll
    for (int n = 0; n < 16; ++n) { acc[n][0] *= corr; acc[n][1] *= corr; }
    const uint32_t pa0 = pack_bf16(sc[0][0], sc[0][1]);
    const uint32_t pa2 = pack_bf16(sc[1][0], sc[1][1]);
    // ---- O += P V  (V^T fragments via ldmatrix.trans)
    {
      const uint32_t row = (lane & 7) + (((lane >> 3) & 1) << 3);
      const uint32_t csel = lane >> 4;
#pragma unroll
      for (int dc = 0; dc < 8; ++dc) {
        const uint32_t half = dc >> 2;
        const uint32_t chunk16 = ((dc & 3) << 1) + csel;
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(vb + half * kHalfBytes + sw128(row, chunk16), v0, v1, v2, v3);
        mma_bf16_16816(acc[2 * dc], pa0, 0u, pa2, 0u, v0, v1);
        mma_bf16_16816(acc[2 * dc + 1], pa0, 0u, pa2, 0u, v2, v3);
      }
    }
    __syncwarp();
    produce(s);  // refill this stage (all lanes finished reading it)

    if (page + 1 == page_end) {
      // ---- item done: finalize
      float l = l_run;
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
      const int nchunks = __ldg(a.ws.prefix + b + 1) - __ldg(a.ws.prefix + b);
      if (r < a.g) {
        const int head = h * a.g + r;
        if (nchunks == 1) {
          const float inv = 1.f / l;
          uint32_t *orow = reinterpret_cast<uint32_t *>(a.out + ((size_t)b * a.Hq + head) * kD);
#pragma unroll
          for (int n = 0; n < 16; ++n) orow[n * 4 + qd] = pack_bf16(acc[n][0] * inv, acc[n][1] * inv);
        } else {
          float2 *orow = reinterpret_cast<float2 *>(a.ws.part_o + ((size_t)chunk * a.Hq + head) * kD);
#pragma unroll
          for (int n = 0; n < 16; ++n) orow[n * 4 + qd] = make_float2(acc[n][0], acc[n][1]);
          if (qd == 0) a.ws.part_ml[(size_t)chunk * a.Hq + head] = make_float2(m_run, l);
        }
      }
    }
  }
  if (fail && lane == 0) atomicExch(a.ws.meta + 3, 1);  // error flag, read by tests
}

// One warp per (sequence, q head): merge the chunk partials of sequences that
// were split; sequences of length 0 get zeros (reference: o = 0 / (0 + eps)).
__global__ void __launch_bounds__(256)
decode_combine_kernel(DecodeArgs a) {
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  // the chunk kernel is done: rewind its work counter, so that a later call
  // on the same stream may reuse this plan (vj_paged_decode_planned)
  if (blockIdx.x == 0 && threadIdx.x == 0) a.ws.meta[2] = 0;
  if (wid >= a.B * a.Hq) return;
  const int b = wid / a.Hq, head = wid % a.Hq;
  const int c0 = a.ws.prefix[b], c1 = a.ws.prefix[b + 1];
  const int n = c1 - c0;
  uint2 *orow = reinterpret_cast<uint2 *>(a.out + ((size_t)b * a.Hq + head) * kD);
  if (n == 1) return;  // written by the chunk kernel
  if (n == 0) { orow[lane] = make_uint2(0u, 0u); return; }
  // m and l of the chunks, lane-parallel
  float M = -INFINITY;
  for (int c = c0 + lane; c < c1; c += 32) M = fmaxf(M, a.ws.part_ml[(size_t)c * a.Hq + head].x);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float L = 0.f;
  for (int c = c0 + lane; c < c1; c += 32) {
    const float2 ml = a.ws.part_ml[(size_t)c * a.Hq + head];
    L += fast_exp2(ml.x - M) * ml.y;
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  // weighted sum of the partial outputs, four chunks in flight
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int c = c0; c < c1; c += 4) {
    float4 p[4];
    float w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bool in = c + j < c1;
      const size_t row = (size_t)(in ? c + j : c0) * a.Hq + head;
      p[j] = reinterpret_cast<const float4 *>(a.ws.part_o + row * kD)[lane];
      w[j] = in ? fast_exp2(a.ws.part_ml[row].x - M) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      o.x += w[j] * p[j].x; o.y += w[j] * p[j].y; o.z += w[j] * p[j].z; o.w += w[j] * p[j].w;
    }
  }
  const float inv = 1.f / (L + 1.1920929e-07f);  // + finfo(f32).eps as at :279-280
  orow[lane] = make_uint2(pack_bf16(o.x * inv, o.y * inv), pack_bf16(o.z * inv, o.w * inv));
}

size_t smem_bytes() {
  return 1024 + kWarps * kStages * (kStageBytes + 8 + 16);
}

}  // namespace
}  // namespace vj

extern "C" size_t vj_paged_decode_workspace_size(int32_t batch, int32_t num_q_heads,
                                                 int32_t head_dim, int32_t max_chunks) {
  if (batch < 0 || num_q_heads <= 0 || head_dim != vj::kD) return 0;
  if (max_chunks <= 0) max_chunks = 4096 + batch;
  return vj::workspace_bytes(batch, num_q_heads, max_chunks);
}

namespace vj {
namespace {
vj_status decode_impl(
    const void *q, const void *k_cache, const void *v_cache, const int32_t *block_tables,
    const int32_t *context_lens, void *out, int32_t batch, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t bt_width, int32_t bt_stride, int64_t stride_block, int64_t stride_token,
    int64_t stride_head, float scale, int32_t max_chunks, void *workspace,
    size_t workspace_bytes, cudaStream_t stream, bool plan);
}  // namespace
}  // namespace vj

extern "C" vj_status vj_paged_decode(
    const void *q, const void *k_cache, const void *v_cache, const int32_t *block_tables,
    const int32_t *context_lens, void *out, int32_t batch, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t bt_width, int32_t bt_stride, int64_t stride_block, int64_t stride_token,
    int64_t stride_head, float scale, int32_t max_chunks, void *workspace,
    size_t workspace_bytes, cudaStream_t stream) {
  return vj::decode_impl(q, k_cache, v_cache, block_tables, context_lens, out, batch,
                         num_q_heads, num_kv_heads, head_dim, num_blocks, block_size, bt_width,
                         bt_stride, stride_block, stride_token, stride_head, scale, max_chunks,
                         workspace, workspace_bytes, stream, true);
}

extern "C" vj_status vj_paged_decode_planned(
    const void *q, const void *k_cache, const void *v_cache, const int32_t *block_tables,
    const int32_t *context_lens, void *out, int32_t batch, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t bt_width, int32_t bt_stride, int64_t stride_block, int64_t stride_token,
    int64_t stride_head, float scale, int32_t max_chunks, void *workspace,
    size_t workspace_bytes, cudaStream_t stream) {
  return vj::decode_impl(q, k_cache, v_cache, block_tables, context_lens, out, batch,
                         num_q_heads, num_kv_heads, head_dim, num_blocks, block_size, bt_width,
                         bt_stride, stride_block, stride_token, stride_head, scale, max_chunks,
                         workspace, workspace_bytes, stream, false);
}

namespace vj {
namespace {
vj_status decode_impl(
    const void *q, const void *k_cache, const void *v_cache, const int32_t *block_tables,
    const int32_t *context_lens, void *out, int32_t batch, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t bt_width, int32_t bt_stride, int64_t stride_block, int64_t stride_token,
    int64_t stride_head, float scale, int32_t max_chunks, void *workspace,
    size_t workspace_bytes, cudaStream_t stream, bool plan) {
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 || bt_width < 0 ||
      bt_stride < bt_width) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_paged_decode: negative or zero size");
  }
  if (num_q_heads % num_kv_heads != 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_paged_decode: Number of Q heads must be divisible by number of KV heads. Got " +
                         std::to_string(num_q_heads) + " and " + std::to_string(num_kv_heads) + ".");
  }
  const int g = num_q_heads / num_kv_heads;
  if (head_dim != kD) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_decode: head_dim must be 128");
  }
  if (g > 8) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_decode: at most 8 query heads per KV head");
  }
  // the chunk kernel's stage words pack (kv head, chunk) as h | chunk << 8
  if (num_kv_heads > 255) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_decode: at most 255 KV heads");
  }
  if (max_chunks >= (1 << 23)) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_decode: max_chunks must be below 2^23");
  }
  if (block_size <= 0 || block_size % kPageTok != 0) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_decode: block_size must be a multiple of 16");
  }
  if (stride_block != (int64_t)block_size * stride_token) {
    return set_error(VJ_ERR_UNSUPPORTED,
                     "vj_paged_decode: tokens of a block must be evenly strided (stride_block == "
                     "block_size * stride_token)");
  }
  if (num_blocks * block_size > (int64_t)INT32_MAX) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_decode: pool larger than 2^31 slots");
  }
  if (batch == 0) return VJ_OK;
  if (!q || !k_cache || !v_cache || !block_tables || !context_lens || !out) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_paged_decode: null pointer");
  }
  if (max_chunks <= 0) max_chunks = 4096 + batch;
  if (max_chunks <= batch) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_paged_decode: max_chunks must exceed batch");
  }
  const size_t need = vj::workspace_bytes(batch, num_q_heads, max_chunks);
  if (!workspace || workspace_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 16 != 0) {
    return set_error(VJ_ERR_WORKSPACE, "vj_paged_decode: workspace needs " + std::to_string(need) +
                                           " bytes, 16-byte aligned");
  }
  CUtensorMap tmk, tmv;
  const uint64_t ntok = (uint64_t)num_blocks * block_size;
  // order the two outer dims by stride (engine layout: heads inside a token row)
  const bool head_major = stride_head < stride_token;
  int rc;
  for (int i = 0; i < 2; ++i) {
    CUtensorMap *m = i ? &tmv : &tmk;
    const void *base = i ? v_cache : k_cache;
    rc = head_major ? encode_tmap_3d(m, base, kD, num_kv_heads, ntok, stride_head * 2,
                                     stride_token * 2, 64, 1, kPageTok, true)
                    : encode_tmap_3d(m, base, kD, ntok, num_kv_heads, stride_token * 2,
                                     stride_head * 2, 64, kPageTok, 1, true);
    if (rc) return rc;
  }

  DecodeArgs a;
  a.q = static_cast<const __nv_bfloat16 *>(q);
  a.out = static_cast<__nv_bfloat16 *>(out);
  a.bt = block_tables;
  a.lens = context_lens;
  a.B = batch; a.Hq = num_q_heads; a.Hkv = num_kv_heads; a.g = g;
  a.bt_stride = bt_stride;
  a.max_pages = bt_width * (block_size / kPageTok);
  a.pages_per_block = block_size / kPageTok;
  a.block_size = block_size;
  a.num_blocks = (int)num_blocks;
  a.head_major = head_major ? 1 : 0;
  a.scale_log2 = scale * kLog2e;
  a.ws = carve(workspace, batch, num_q_heads, max_chunks);

  const int grid = num_sms() * kCtasPerSm;
  if (plan) {
    decode_plan_kernel<<<1, 1024, 0, stream>>>(context_lens, batch, num_kv_heads, max_chunks,
                                               grid * kWarps, a.max_pages, a.ws);
    rc = check_launch("vj_paged_decode(plan)");
    if (rc) return rc;
  }
  const size_t smem = smem_bytes();
  cudaFuncSetAttribute(decode_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  decode_chunk_kernel<<<grid, kWarps * 32, smem, stream>>>(tmk, tmv, a);
  rc = check_launch("vj_paged_decode(chunks)");
  if (rc) return rc;
  const int warps = batch * num_q_heads;
  decode_combine_kernel<<<(warps + 7) / 8, 256, 0, stream>>>(a);
  return check_launch("vj_paged_decode(combine)");
}
}  // namespace
}  // namespace vj

// ---------------------------------------------------------------------------
// Decode for callers that cannot allocate device memory.
//
// Some callers may not call cudaMalloc at all: a custom-call handler inside
// an XLA / JAX computation, where the runtime owns every device buffer and an
// allocation inside the handler would bypass its accounting and may
// synchronise the device, or a serving process that pins its whole memory
// budget at start-up. vj_paged_decode_noalloc takes the same inputs and
// outputs as vj_paged_decode but keeps its split-KV scratch in a fixed
// file-scope device array instead of a caller workspace.
//
// The array (kStaticScratchBytes) exists on every GPU that loads this
// library and stays allocated until the process exits. All calls on a device
// share it and it keeps the previous call's contents; the plan kernel
// rewrites every word a call reads before it is read, so nothing needs
// clearing, but two calls whose kernels overlap on the GPU (different
// streams, no ordering between them) race on the array.
// ---------------------------------------------------------------------------
namespace vj {
namespace {
constexpr size_t kStaticScratchBytes = size_t(16) << 20;  // 16 MiB per device
__device__ __align__(256) uint8_t g_decode_scratch[kStaticScratchBytes];

// The array's address belongs to a CUDA context (a module is loaded per
// context), so the cache is keyed by the current context; with the runtime's
// primary contexts that is once per device. The lookup makes no allocation.
constexpr int kMaxContexts = 128;
std::mutex g_scratch_mu;
struct ScratchEntry {
  CUcontext ctx;
  void *ptr;
};
ScratchEntry g_scratch_cache[kMaxContexts];
int g_scratch_entries = 0;
using CtxGetCurrentFn = CUresult (*)(CUcontext *);
CtxGetCurrentFn g_ctx_get_current = nullptr;

// Device address of g_decode_scratch in the current context. In host code the
// symbol only names a host-side stand-in, so the address is looked up once
// per context (with it current) and cached.
int scratch_address(void **ptr) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_ctx_get_current == nullptr) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr) {
      return set_error(VJ_ERR_CUDA, "vj_paged_decode_noalloc: cuCtxGetCurrent not found");
    }
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
  }
  CUcontext ctx = nullptr;
  void *p = nullptr;
  cudaError_t e = cudaSuccess;
  if (g_ctx_get_current(&ctx) != CUDA_SUCCESS) {
    return set_error(VJ_ERR_CUDA, "vj_paged_decode_noalloc: cuCtxGetCurrent failed");
  }
  if (ctx == nullptr) {
    // no context on this thread yet: the runtime call below creates and binds
    // the device's primary context
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || g_ctx_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
      return set_error(VJ_ERR_CUDA, "vj_paged_decode_noalloc: no CUDA context");
    }
  }
  for (int i = 0; i < g_scratch_entries; ++i) {
    if (g_scratch_cache[i].ctx == ctx) {
      *ptr = g_scratch_cache[i].ptr;
      return VJ_OK;
    }
  }
  if (g_scratch_entries == kMaxContexts) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_decode_noalloc: too many CUDA contexts");
  }
  if (p == nullptr) e = cudaGetSymbolAddress(&p, g_decode_scratch);
  if (e != cudaSuccess || p == nullptr) {
    return set_error(VJ_ERR_CUDA, std::string("vj_paged_decode_noalloc: cudaGetSymbolAddress: ") +
                                      cudaGetErrorString(e));
  }
  g_scratch_cache[g_scratch_entries++] = {ctx, p};
  *ptr = p;
  return VJ_OK;
}
}  // namespace
}  // namespace vj

extern "C" size_t vj_paged_decode_noalloc_scratch_bytes(void) { return vj::kStaticScratchBytes; }

extern "C" vj_status vj_paged_decode_noalloc(
    const void *q, const void *k_cache, const void *v_cache, const int32_t *block_tables,
    const int32_t *context_lens, void *out, int32_t batch, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t bt_width, int32_t bt_stride, int64_t stride_block, int64_t stride_token,
    int64_t stride_head, float scale, cudaStream_t stream) {
  using namespace vj;
  if (batch < 0 || num_q_heads <= 0 || head_dim != kD) {
    // let the shared entry point produce its usual argument message
    return vj_paged_decode(q, k_cache, v_cache, block_tables, context_lens, out, batch,
                           num_q_heads, num_kv_heads, head_dim, num_blocks, block_size, bt_width,
                           bt_stride, stride_block, stride_token, stride_head, scale, 0, nullptr,
                           0, stream);
  }
  // Largest split budget whose scratch fits the fixed array.
  const size_t per_chunk = (size_t)num_q_heads * (sizeof(float2) + sizeof(float) * kD);
  int64_t max_chunks = (int64_t)(kStaticScratchBytes / per_chunk);
  while (max_chunks > 0 &&
         vj::workspace_bytes(batch, num_q_heads, (int)max_chunks) > kStaticScratchBytes) {
    --max_chunks;
  }
  if (max_chunks <= batch) {
    return set_error(VJ_ERR_UNSUPPORTED,
                     "vj_paged_decode_noalloc: batch " + std::to_string(batch) + " with " +
                         std::to_string(num_q_heads) + " query heads needs more than the " +
                         std::to_string(kStaticScratchBytes >> 20) +
                         " MiB fixed scratch (at most " + std::to_string(max_chunks - 1) +
                         " sequences at this head count); use vj_paged_decode with a workspace");
  }
  void *scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  return vj_paged_decode(q, k_cache, v_cache, block_tables, context_lens, out, batch,
                         num_q_heads, num_kv_heads, head_dim, num_blocks, block_size, bt_width,
                         bt_stride, stride_block, stride_token, stride_head, scale,
                         (int32_t)max_chunks, scratch, kStaticScratchBytes, stream);
}
