// K1: varlen paged prefill attention on 5th-gen tensor cores (tcgen05 + TMEM),
// fed by TMA straight from the paged KV pool.
//
// Replaces vllm/kernels/prefill_paged_attention.py:407-453
// (prefill_paged_attention -> _unbatched :160-388, Pallas kernel :18-150),
// including its Q gather (:227-239), split-KV merge (:364-376) and scatter
// back to packed token order (:384-388), and generalises it to a cached
// prefix: new token i of sequence s sits at position ctx_s - n_s + i and
// attends to keys [0, that position].
//
// One CTA = one 128-row Q tile of one (sequence, KV head): the rows pack the
// GQA group, row r = (token r / g, head r % g), so each K/V byte loaded by TMA
// feeds all g query heads. Keys stream in tiles of 128 (8 pages of 16).
// Both GEMMs take their A operand from tensor memory, so shared memory only
// feeds B (K or V) and the tensor pipe is not capped by smem bandwidth:
//   TMEM columns [0,128) S0 | [128,256) S1 | [256,384) O | [384,448) Q
//   P_j (bf16) overwrites the first 64 columns of S_(j&1) after softmax reads it.
// Warp roles (192 threads):
//   warps 0-3  softmax: one thread per row. Loads its Q row into TMEM once;
//              per key tile reads S from TMEM, online softmax in fp32 (exp2),
//              writes P back into TMEM, and rescales O in TMEM only when the
//              running max grows by more than 2^8 (exact: l and O always
//              share the same reference max)
//   warp 4     TMA producer: K/V pages through a 3-stage ring
//   warp 5     MMA issuer (one thread), in order QK_0, QK_1, PV_0, QK_2, PV_1
//              ...: S_(j+1) is computed while softmax works on S_j
// Tensor-core bound: FLOPs = 4 * Hq * D * (n*p + n(n+1)/2) per sequence.
#include "../../include/vjattn.h"
#include "vj_common.cuh"

#include <string>

namespace vj {
namespace {

constexpr int kD = 128;
constexpr int kBM = 128;   // rows per Q tile
constexpr int kBN = 128;   // keys per KV tile
constexpr int kPageTok = 16;
constexpr int kPagesPerTile = kBN / kPageTok;
constexpr int kThreads = 192;
constexpr int kHalf = 128 * 128;   // bytes of a [128 rows x 64 bf16] swizzled half tile
constexpr int kTile = 2 * kHalf;   // [128 x 128] bf16
constexpr int kStages = 3;
constexpr int OFF_K = 0;
constexpr int OFF_V = OFF_K + kStages * kTile;
constexpr int OFF_BAR = OFF_V + kStages * kTile;
constexpr uint32_t TM_S = 0, TM_O = 256, TM_Q = 384;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr float kLog2e = 1.4426950408889634f;

struct Bars {
  uint64_t q_full;
  uint64_t k_full[kStages], k_empty[kStages], v_full[kStages], v_empty[kStages];
  uint64_t s_full[2];
  uint64_t p_full, o_done;
  uint32_t tmem_base;
  int abort;
};
constexpr size_t kSmemBytes = 1024 + OFF_BAR + sizeof(Bars);

struct PrefillArgs {
  const __nv_bfloat16 *q;
  __nv_bfloat16 *out;
  const int32_t *bt;
  const int32_t *cu;
  const int32_t *ctx_lens;  // may be null: keys == new tokens
  int Hq, Hkv, g, tt;       // tt = tokens per Q tile = 128 / g
  int bt_stride, max_pages, pages_per_block, block_size, num_blocks;
  int head_major;
  int num_tokens;
  float scale_log2;
  int *err;
};

// Token coordinate (flat pool token index of the page's first token) of page
// grp*32 + lane of sequence s: one coalesced block-table read per 4 KV tiles.
VJ_DEV int page_tok0(const PrefillArgs &a, const int32_t *row, int grp, int lane) {
  const int page = grp * 32 + lane;
  int blk = 0;
  if (page < a.max_pages) {
    blk = __ldg(row + page / a.pages_per_block);
    if (blk < 0 || blk >= a.num_blocks) blk = 0;  // safe_block_tables
  }
  return blk * a.block_size + (page % a.pages_per_block) * kPageTok;
}

// Issue the 16 TMA boxes (8 pages x 2 dim halves) of one K or V tile; the
// page coordinates live in the producer warp's lanes (tile jj of the group).
VJ_DEV void load_kv_tile(const CUtensorMap *tm, uint8_t *dst, uint64_t *bar, const PrefillArgs &a,
                         int h, int toks, int jj, int lane) {
#pragma unroll
  for (int pg = 0; pg < kPagesPerTile; ++pg) {
    const int tok0 = __shfl_sync(0xffffffffu, toks, jj * kPagesPerTile + pg);
    if (lane == 0) {
      const int c1 = a.head_major ? h : tok0, c2 = a.head_major ? tok0 : h;
      tma_load_3d(dst + pg * (kPageTok * 128), tm, bar, 0, c1, c2);
      tma_load_3d(dst + kHalf + pg * (kPageTok * 128), tm, bar, 64, c1, c2);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
prefill_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
               PrefillArgs a) {
  const int s = blockIdx.z, h = blockIdx.y;
  const int m = gridDim.x - 1 - blockIdx.x;  // longest tiles first
  const int q0 = __ldg(a.cu + s);
  const int n = __ldg(a.cu + s + 1) - q0;
  const int tq0 = m * a.tt;
  if (tq0 >= n) return;  // whole CTA, before any barrier or TMEM use
  int ctx = a.ctx_lens ? __ldg(a.ctx_lens + s) : n;
  if (ctx < n) ctx = n;
  const int p0 = ctx - n;                          // cached prefix length
  const int qpos_min = p0 + tq0;
  const int kv_end = p0 + min(n, tq0 + a.tt);      // keys visible to the last row
  const int nkv = (kv_end + kBN - 1) / kBN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  Bars &bar = *reinterpret_cast<Bars *>(smem + OFF_BAR);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bar.q_full, 128);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&bar.k_full[i], 1);
      mbar_init(&bar.k_empty[i], 1);
      mbar_init(&bar.v_full[i], 1);
      mbar_init(&bar.v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) mbar_init(&bar.s_full[i], 1);
    mbar_init(&bar.p_full, 128);
    mbar_init(&bar.o_done, 1);
    bar.abort = 0;
    fence_mbar_init();
  }
  if (warp == 5) tmem_alloc(&bar.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem_base;
  bool ok = true;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    // whole warp: lanes hold page coordinates, lane 0 issues the copies
    const int32_t *row = a.bt + (size_t)s * a.bt_stride;
    int cur = page_tok0(a, row, 0, lane);
    int nxt = nkv > 4 ? page_tok0(a, row, 1, lane) : 0;
    if (lane == 0) { tma_prefetch_desc(&tmk); tma_prefetch_desc(&tmv); }
    for (int j = 0; j < nkv && ok; ++j) {
      const int st = j % kStages, jj = j & 3;
      const uint32_t use = j / kStages;  // how many times this stage was filled before
      if (jj == 0 && j > 0) {
        cur = nxt;
        nxt = j + 4 < nkv ? page_tok0(a, row, (j >> 2) + 1, lane) : 0;
      }
      if (use > 0) ok = mbar_wait(&bar.k_empty[st], (use - 1) & 1);
      if (!ok) break;
      if (lane == 0) mbar_arrive_expect_tx(&bar.k_full[st], kTile);
      load_kv_tile(&tmk, smem + OFF_K + st * kTile, &bar.k_full[st], a, h, cur, jj, lane);
      if (use > 0) ok = mbar_wait(&bar.v_empty[st], (use - 1) & 1);
      if (!ok) break;
      if (lane == 0) mbar_arrive_expect_tx(&bar.v_full[st], kTile);
      load_kv_tile(&tmv, smem + OFF_V + st * kTile, &bar.v_full[st], a, h, cur, jj, lane);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = umma_idesc_bf16(kBM, kBN, false);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(kBM, kD, true);
      const uint32_t sk = smem_u32(smem + OFF_K), sv = smem_u32(smem + OFF_V);
      auto issue_qk = [&](int j) -> bool {
        const int st = j % kStages;
        if (!mbar_wait(&bar.k_full[st], (j / kStages) & 1)) return false;
        tc_fence_after();
        const uint32_t kb = sk + st * kTile;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          // A = Q (TMEM, 8 columns per 16 dims), B = K tile (K-major, swizzled)
          umma_ts(tmem + TM_S + (j & 1) * kBN, tmem + TM_Q + kk * 8,
                  umma_desc_sw128(kb + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024), idesc_qk,
                  kk > 0 ? 1u : 0u);
        }
        umma_commit(&bar.s_full[j & 1]);
        umma_commit(&bar.k_empty[st]);
        return true;
      };
      ok = mbar_wait(&bar.q_full, 0);
      tc_fence_after();
      if (ok) ok = issue_qk(0);
      for (int j = 0; j < nkv && ok; ++j) {
        // S_(j+1) overwrites the buffer of P_(j-1); PV_(j-1) was issued
        // before it and tcgen05 MMAs of one thread execute in issue order.
        if (j + 1 < nkv) {
          ok = issue_qk(j + 1);
          if (!ok) break;
        }
        const int st = j % kStages;
        ok = mbar_wait(&bar.p_full, j & 1);
        if (ok) ok = mbar_wait(&bar.v_full[st], (j / kStages) & 1);
        if (!ok) break;
        tc_fence_after();
        const uint32_t vb = sv + st * kTile;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          // A = P (TMEM, aliased on S_(j&1)), B = V tile (MN-major: keys x dims)
          umma_ts(tmem + TM_O, tmem + TM_S + (j & 1) * kBN + kk * 8,
                  umma_desc_sw128(vb + kk * 2048, kHalf, 1024), idesc_pv,
                  (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bar.o_done);
        umma_commit(&bar.v_empty[st]);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int r = threadIdx.x;  // row of the Q tile == TMEM lane
    const int tq = tq0 + r / a.g;
    const int qpos = p0 + tq;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    {
      // this row of Q -> TMEM (two bf16 per column); rows past the tensor are 0
      uint32_t qv[64];
      const int64_t tok = (int64_t)q0 + tq;
      if (tok < a.num_tokens) {
        const uint4 *src = reinterpret_cast<const uint4 *>(
            a.q + (tok * a.Hq + (int64_t)h * a.g + (r % a.g)) * kD);
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const uint4 w = __ldg(src + c);
          qv[4 * c] = w.x; qv[4 * c + 1] = w.y; qv[4 * c + 2] = w.z; qv[4 * c + 3] = w.w;
        }
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) qv[c] = 0u;
      }
      tmem_st64_sync(tmem + lane_base + TM_Q, qv);
      tc_fence_before();
      mbar_arrive(&bar.q_full);
    }
    float m_run = -INFINITY, l_run = 0.f;
    float sv[kBN];
    for (int j = 0; j < nkv; ++j) {
      const int b = j & 1;
      ok = mbar_wait(&bar.s_full[b], (j >> 1) & 1);
      if (!ok) break;
      tc_fence_after();
      tmem_ld128(tmem + lane_base + TM_S + b * kBN, sv);

      const int kbase = j * kBN;
      const bool masked = kbase + kBN - 1 > qpos_min;
      float mx = -INFINITY;
      if (masked) {
#pragma unroll
        for (int i = 0; i < kBN; ++i) {
          if (kbase + i > qpos) sv[i] = -INFINITY;
          mx = fmaxf(mx, sv[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < kBN; ++i) mx = fmaxf(mx, sv[i]);
      }
      // scores are raw q.k; the softmax scale (and log2 e) folds into one FFMA
      const float m_new = fmaxf(m_run, mx * a.scale_log2);
      const bool need = j > 0 && (m_new - m_run > kRescaleThreshold);
      const float m_use = (j == 0 || need) ? m_new : m_run;
      const float corr = j == 0 ? 0.f : fast_exp2(m_run - m_use);
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < kBN; ++i) {
        sv[i] = fast_exp2(fmaf(sv[i], a.scale_log2, -m_use));
        sum += sv[i];
      }
      l_run = l_run * corr + sum;
      m_run = m_use;

      if (j >= 1) {
        ok = mbar_wait(&bar.o_done, (j - 1) & 1);
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int c = 0; c < kD / 32; ++c) {
            float t[32];
            const uint32_t ta = tmem + lane_base + TM_O + c * 32;
            tmem_ld32(ta, t);
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] *= corr;
            tmem_st32(ta, t);
          }
          tmem_st_wait();
        }
      }
      // P row r (bf16 pairs) -> TMEM over the first 64 columns of S_b
      {
        uint32_t pv[64];
#pragma unroll
        for (int c = 0; c < 64; ++c) pv[c] = pack_bf16(sv[2 * c], sv[2 * c + 1]);
        tmem_st64_sync(tmem + lane_base + TM_S + b * kBN, pv);
      }
      tc_fence_before();
      mbar_arrive(&bar.p_full);
    }
    // ---- epilogue: O / l -> bf16 rows of the packed output
    if (ok) ok = mbar_wait(&bar.o_done, (nkv - 1) & 1);
    if (ok) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      const bool valid = tq < n && q0 + tq < a.num_tokens;
      __nv_bfloat16 *orow =
          a.out + ((size_t)(q0 + tq) * a.Hq + (size_t)h * a.g + (r % a.g)) * kD;
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        float t[32];
        tmem_ld32(tmem + lane_base + TM_O + c * 32, t);
        if (valid) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            w.x = pack_bf16(t[i] * inv, t[i + 1] * inv);
            w.y = pack_bf16(t[i + 2] * inv, t[i + 3] * inv);
            w.z = pack_bf16(t[i + 4] * inv, t[i + 5] * inv);
            w.w = pack_bf16(t[i + 6] * inv, t[i + 7] * inv);
            *reinterpret_cast<uint4 *>(orow + c * 32 + i) = w;
          }
        }
      }
    }
  }
  if (!ok) atomicExch(a.err, 1);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, 512);
}

// Rows of the packed output past cu_seqlens_q[num_seqs] (bucket padding) -> 0,
// as the reference's scatter leaves them (prefill_paged_attention.py:384-388).
__global__ void prefill_zero_tail_kernel(__nv_bfloat16 *out, const int32_t *cu, int num_seqs,
                                         int64_t num_tokens, int row_elems) {
  const int64_t start = (int64_t)__ldg(cu + num_seqs) * row_elems;
  const int64_t end = num_tokens * row_elems;
  uint4 *o = reinterpret_cast<uint4 *>(out);
  for (int64_t i = start / 8 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < end / 8;
       i += (int64_t)gridDim.x * blockDim.x) {
    o[i] = make_uint4(0u, 0u, 0u, 0u);
  }
}

}  // namespace
}  // namespace vj

extern "C" vj_status vj_paged_prefill(
    const void *q, const void *k_cache, const void *v_cache, const int32_t *block_tables,
    const int32_t *cu_seqlens_q, const int32_t *context_lens, void *out, int64_t num_tokens,
    int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
    int64_t num_blocks, int32_t block_size, int32_t bt_width, int32_t bt_stride,
    int64_t stride_block, int64_t stride_token, int64_t stride_head, int32_t max_seqlen_q,
    float scale, int32_t *error_flag, cudaStream_t stream) {
  using namespace vj;
  if (num_tokens < 0 || num_seqs < 0 || num_q_heads <= 0 || num_kv_heads <= 0 ||
      num_blocks <= 0 || bt_width < 0 || bt_stride < bt_width) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_paged_prefill: negative or zero size");
  }
  if (num_q_heads % num_kv_heads != 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_paged_prefill: Number of Q heads must be divisible by number of KV "
                     "heads. Got " + std::to_string(num_q_heads) + " and " +
                         std::to_string(num_kv_heads) + ".");
  }
  const int g = num_q_heads / num_kv_heads;
  if (head_dim != kD) return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_prefill: head_dim must be 128");
  if (kBM % g != 0) {
    return set_error(VJ_ERR_UNSUPPORTED,
                     "vj_paged_prefill: query heads per KV head must divide 128");
  }
  if (block_size <= 0 || block_size % kPageTok != 0) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_prefill: block_size must be a multiple of 16");
  }
  if (stride_block != (int64_t)block_size * stride_token) {
    return set_error(VJ_ERR_UNSUPPORTED,
                     "vj_paged_prefill: stride_block must equal block_size * stride_token");
  }
  if (num_blocks * block_size > (int64_t)INT32_MAX || num_tokens > (int64_t)INT32_MAX) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_prefill: sizes beyond 2^31");
  }
  if (num_tokens == 0) return VJ_OK;
  if (!q || !k_cache || !v_cache || !cu_seqlens_q || !out || !error_flag ||
      (num_seqs > 0 && !block_tables)) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_paged_prefill: null pointer");
  }
  const int tt = kBM / g;
  CUtensorMap tmk, tmv;
  int rc = VJ_OK;
  const uint64_t ntok = (uint64_t)num_blocks * block_size;
  const bool head_major = stride_head < stride_token;
  for (int i = 0; i < 2; ++i) {
    CUtensorMap *mp = i ? &tmv : &tmk;
    const void *base = i ? v_cache : k_cache;
    rc = head_major ? encode_tmap_3d(mp, base, kD, num_kv_heads, ntok, stride_head * 2,
                                     stride_token * 2, 64, 1, kPageTok, true)
                    : encode_tmap_3d(mp, base, kD, ntok, num_kv_heads, stride_token * 2,
                                     stride_head * 2, 64, kPageTok, 1, true);
    if (rc) return rc;
  }
  PrefillArgs a;
  a.q = static_cast<const __nv_bfloat16 *>(q);
  a.out = static_cast<__nv_bfloat16 *>(out);
  a.bt = block_tables;
  a.cu = cu_seqlens_q;
  a.ctx_lens = context_lens;
  a.Hq = num_q_heads; a.Hkv = num_kv_heads; a.g = g; a.tt = tt;
  a.bt_stride = bt_stride;
  a.pages_per_block = block_size / kPageTok;
  a.max_pages = bt_width * a.pages_per_block;
  a.block_size = block_size;
  a.num_blocks = (int)num_blocks;
  a.head_major = head_major ? 1 : 0;
  a.num_tokens = (int)num_tokens;
  a.scale_log2 = scale * kLog2e;
  a.err = error_flag;

  const int64_t maxq = max_seqlen_q > 0 ? max_seqlen_q : num_tokens;
  const int64_t mtiles = (maxq + tt - 1) / tt;
  if (num_seqs > 0 && mtiles > 0) {
    if (mtiles > INT32_MAX || num_kv_heads > 65535 || num_seqs > 65535) {
      return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_prefill: grid too large");
    }
    cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)kSmemBytes);
    dim3 grid((unsigned)mtiles, num_kv_heads, num_seqs);
    prefill_kernel<<<grid, kThreads, kSmemBytes, stream>>>(tmk, tmv, a);
    rc = check_launch("vj_paged_prefill");
    if (rc) return rc;
  }
  prefill_zero_tail_kernel<<<num_sms() * 2, 256, 0, stream>>>(
      static_cast<__nv_bfloat16 *>(out), cu_seqlens_q, num_seqs, num_tokens, num_q_heads * kD);
  return check_launch("vj_paged_prefill(zero tail)");
}
