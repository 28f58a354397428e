// Device side of K2 (split-KV paged decode attention), shared by the decode
// launches (decode.cu) and the mixed decode + prefill launch (prefill.cu):
// constants, the caller-sized workspace layout, the plan kernel, the body
// of one decode warp and the combine kernel. Included inside
// `namespace vj { namespace { namespace dk {` so that every translation unit
// keeps its own internal copy.
#pragma once

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

// The work of one decode warp: pull (chunk, kv head) items until the queue
// drains. NW decode warps share a CTA's shared memory (1024-byte aligned
// `smem`, smem_bytes(NW)); every warp owns its ring and barriers.
template <int NW>
__device__ __forceinline__ void decode_chunk_body(const CUtensorMap *tmk_p,
                                                  const CUtensorMap *tmv_p, const DecodeArgs &a,
                                                  uint8_t *smem, int warp, int lane) {
  uint8_t *ring = smem + warp * (kStages * kStageBytes);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + NW * kStages * kStageBytes) +
                   warp * kStages;
  // per stage: item id of the page it holds (-1 = drained), page index
  int *st_item = reinterpret_cast<int *>(full + (NW - warp) * kStages) +
                 warp * kStages * 4;

  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    if (warp == 0) { tma_prefetch_desc(tmk_p); tma_prefetch_desc(tmv_p); }
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
        tma_load_3d(dst, tmk_p, &full[s], 0, c1, c2);
        tma_load_3d(dst + kHalfBytes, tmk_p, &full[s], 64, c1, c2);
        tma_load_3d(dst + 2 * kHalfBytes, tmv_p, &full[s], 0, c1, c2);
        tma_load_3d(dst + 3 * kHalfBytes, tmv_p, &full[s], 64, c1, c2);
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

// Shared memory of a CTA with NW decode warps (+1024 for alignment).
constexpr size_t smem_bytes(int nw) {
  return 1024 + (size_t)nw * kStages * (kStageBytes + 8 + 16);
}
