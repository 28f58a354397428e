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
// One CTA = two consecutive 128-row Q tiles (A, B) of one (sequence, KV
// head). Rows pack the GQA group, row r = (token r / g, head r % g), so each
// K/V byte loaded feeds all g query heads of 2 tiles: the paged K/V stream
// (16 TMA boxes of 16 tokens x 64 dims per 128-key tile) is what bounds a
// one-tile-per-CTA design, and sharing it between two tiles halves it.
//
//   TMEM columns: [0,128) S_A | [128,256) S_B | [256,384) O_A | [384,512) O_B
//   P_X (bf16 pairs) overwrites the first 64 columns of S_X after softmax
//   reads it; PV takes P straight from TMEM (A operand), V from smem.
//   Shared memory: Q_A, Q_B (32 KB each), K ring 3 x 32 KB, V ring 2 x 32 KB,
//   all 128-byte swizzled K-major / MN-major UMMA layouts written by TMA.
//
// Warp roles (352 threads):
//   warps 0-3 / 4-7  softmax of tile A / B: one thread per row; per key tile
//                    read S (128 fp32 columns) from TMEM, online softmax in
//                    fp32 with exp2 (row max with three-input max.f32, scale
//                    and sums on packed f32x2 ops), P back to TMEM; O is rescaled
//                    in TMEM only when the running max grows by more than
//                    2^8 (exact: l and O always share the same reference max)
//   warp 8           TMA producer of K tiles (and Q once)
//   warp 9           MMA issuer (one thread), order per key tile j:
//                    PV_A(j), QK_A(j+1), PV_B(j), QK_B(j+1) -- the tensor
//                    core works on one tile while softmax works on the other
//   warp 10          TMA producer of V tiles
// Tensor-core bound: FLOPs = 4 * Hq * D * (n*p + n(n+1)/2) per sequence.
#include "../../include/vjattn.h"
#include "vj_common.cuh"

#include <algorithm>
#include <string>

namespace vj {
namespace {
namespace dk {
#include "decode_core.cuh"
}  // namespace dk
}  // namespace
}  // namespace vj

namespace vj {
namespace {

constexpr int kD = 128;
constexpr int kBM = 128;   // rows per Q tile
constexpr int kBN = 128;   // keys per KV tile
constexpr int kPageTok = 16;
constexpr int kPagesPerTile = kBN / kPageTok;
constexpr int kThreads = 352;
constexpr int kWarpK = 8, kWarpMma = 9, kWarpV = 10;
constexpr int kHalf = 128 * 128;   // bytes of a [128 rows x 64 bf16] swizzled half tile
constexpr int kTile = 2 * kHalf;   // [128 x 128] bf16
constexpr int kKStages = 3, kVStages = 2;
constexpr int OFF_Q = 0;                        // Q_A, Q_B
constexpr int OFF_K = OFF_Q + 2 * kTile;
constexpr int OFF_V = OFF_K + kKStages * kTile;
constexpr int OFF_BAR = OFF_V + kVStages * kTile;
constexpr uint32_t TM_S = 0, TM_O = 256;        // + tile * 128
constexpr float kRescaleThreshold = 8.0f;       // log2 units
constexpr float kLog2e = 1.4426950408889634f;

// Softmax exponentials run on the MUFU unit (ex2.approx). Bit k of kEmuMask
// set moves the columns i with i % 8 == k onto a cubic polynomial on the FMA
// pipe instead (2^f on [-0.5, 0.5], fitted for minimum relative error, max
// 2.1e-4, below bf16's 2^-9 rounding of P). Measured on C2 with the packed
// fp32 softmax arithmetic: 990 TFLOP/s with no column on the polynomial, 939
// with 1 of 8, 849 and 722 with 2 and 4 of 8 (before packing): the softmax
// threads are bound by issue, not by MUFU, so the default moves none.
#ifndef VJ_PREFILL_EMU_MASK
#define VJ_PREFILL_EMU_MASK 0x00
#endif
constexpr unsigned kEmuMask = VJ_PREFILL_EMU_MASK;
constexpr float kP0 = 0.99995905f, kP1 = 0.69357258f, kP2 = 0.24221395f, kP3 = 0.05302752f;

// max of three (sm_100 three-input max.f32; exact, like two fmaxf)
VJ_DEV float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

VJ_DEV float poly_exp2(float x) {
  x = fmaxf(x, -125.f);                  // keeps the exponent field positive
  const float t = x + 12582912.f;        // 1.5 * 2^23: round(x) lands in the low bits
  const float n = t - 12582912.f;
  const float f = x - n;                 // [-0.5, 0.5]
  const float p = fmaf(fmaf(fmaf(kP3, f, kP2), f, kP1), f, kP0);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

struct Bars {
  uint64_t q_full;
  uint64_t k_full[kKStages], k_empty[kKStages];
  uint64_t v_full[kVStages], v_empty[kVStages];
  uint64_t s_full[2], p_full[2], o_final[2];
  uint32_t tmem_base;
};
constexpr size_t kSmemBytes = 1024 + OFF_BAR + sizeof(Bars);
static_assert(kSmemBytes <= 232448, "shared memory budget");

struct PrefillArgs {
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

// Stream the K or V tiles of one work item through a ring of `stages`
// buffers; the whole warp runs this (lanes hold page coordinates), lane 0
// issues the copies. Returns false if a wait timed out.
template <int kStagesT>
VJ_DEV bool produce_kv(const CUtensorMap *tm, uint8_t *ring, uint64_t *full, uint64_t *empty,
                       const PrefillArgs &a, int s, int h, int nkv, int lane) {
  const int32_t *row = a.bt + (size_t)s * a.bt_stride;
  int cur = page_tok0(a, row, 0, lane);
  int nxt = nkv > 4 ? page_tok0(a, row, 1, lane) : 0;
  for (int j = 0; j < nkv; ++j) {
    const int st = j % kStagesT, jj = j & 3;
    const int use = j / kStagesT;
    if (jj == 0 && j > 0) {
      cur = nxt;
      nxt = j + 4 < nkv ? page_tok0(a, row, (j >> 2) + 1, lane) : 0;
    }
    bool ok = true;
    if (use > 0) ok = mbar_wait(&empty[st], (use - 1) & 1);
    if (!__all_sync(0xffffffffu, ok)) return false;
    if (lane == 0) mbar_arrive_expect_tx(&full[st], kTile);
    uint8_t *dst = ring + st * kTile;
#pragma unroll
    for (int pg = 0; pg < kPagesPerTile; ++pg) {
      const int tok0 = __shfl_sync(0xffffffffu, cur, jj * kPagesPerTile + pg);
      if (lane == 0) {
        const int c1 = a.head_major ? h : tok0, c2 = a.head_major ? tok0 : h;
        tma_load_3d(dst + pg * (kPageTok * 128), tm, &full[st], 0, c1, c2);
        tma_load_3d(dst + kHalf + pg * (kPageTok * 128), tm, &full[st], 64, c1, c2);
      }
    }
  }
  return true;
}

// The work of one CTA: tile pair m2 of (sequence s, kv head h). All 352
// threads of the CTA run it.
__device__ __forceinline__ void prefill_body(const CUtensorMap *tmq_p, const CUtensorMap *tmk_p,
                                             const CUtensorMap *tmv_p, const PrefillArgs &a,
                                             int s, int h, int m2, uint8_t *smem_raw) {
  const int q0 = __ldg(a.cu + s);
  const int n = __ldg(a.cu + s + 1) - q0;
  const int tq0 = m2 * 2 * a.tt;               // first token of tile A
  if (tq0 >= n) return;  // whole CTA, before any barrier or TMEM use
  int ctx = a.ctx_lens ? __ldg(a.ctx_lens + s) : n;
  if (ctx < n) ctx = n;
  const int p0 = ctx - n;                          // cached prefix length
  const int kv_end = p0 + min(n, tq0 + 2 * a.tt);  // keys visible to the last row of B
  const int nkv = (kv_end + kBN - 1) / kBN;

  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  Bars &bar = *reinterpret_cast<Bars *>(smem + OFF_BAR);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bar.q_full, 1);
    for (int i = 0; i < kKStages; ++i) { mbar_init(&bar.k_full[i], 1); mbar_init(&bar.k_empty[i], 1); }
    for (int i = 0; i < kVStages; ++i) { mbar_init(&bar.v_full[i], 1); mbar_init(&bar.v_empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar.s_full[i], 1);
      mbar_init(&bar.p_full[i], kBM);
      mbar_init(&bar.o_final[i], 1);
    }
    fence_mbar_init();
  }
  if (warp == kWarpMma) tmem_alloc(&bar.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem_base;
  bool ok = true;

  if (warp == kWarpK) {
    // ------------------------------------------------------------ Q + K producer
    if (lane == 0) {
      tma_prefetch_desc(tmq_p); tma_prefetch_desc(tmk_p); tma_prefetch_desc(tmv_p);
      mbar_arrive_expect_tx(&bar.q_full, 2 * kTile);
      for (int t = 0; t < 2; ++t) {
        const int tok = q0 + tq0 + t * a.tt;
        tma_load_3d(smem + OFF_Q + t * kTile, tmq_p, &bar.q_full, 0, h * a.g, tok);
        tma_load_3d(smem + OFF_Q + t * kTile + kHalf, tmq_p, &bar.q_full, 64, h * a.g, tok);
      }
    }
    ok = produce_kv<kKStages>(tmk_p, smem + OFF_K, bar.k_full, bar.k_empty, a, s, h, nkv, lane);
  } else if (warp == kWarpV) {
    // ------------------------------------------------------------ V producer
    ok = produce_kv<kVStages>(tmv_p, smem + OFF_V, bar.v_full, bar.v_empty, a, s, h, nkv, lane);
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = umma_idesc_bf16(kBM, kBN, false);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(kBM, kD, true);
      const uint32_t sq = smem_u32(smem + OFF_Q), sk = smem_u32(smem + OFF_K),
                     sv = smem_u32(smem + OFF_V);
      // S_t = Q_t K_j^T (both operands from smem, K-major)
      auto qk = [&](int t, int j) {
        const uint32_t kb = sk + (j % kKStages) * kTile, qb = sq + t * kTile;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
          umma_ss(tmem + TM_S + t * kBM, umma_desc_sw128(qb + off, 16, 1024),
                  umma_desc_sw128(kb + off, 16, 1024), idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bar.s_full[t]);
      };
      // O_t += P_t V_j (P from TMEM over S_t, V MN-major in smem)
      auto pv = [&](int t, int j) {
        const uint32_t vb = sv + (j % kVStages) * kTile;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          umma_ts(tmem + TM_O + t * kBM, tmem + TM_S + t * kBM + kk * 8,
                  umma_desc_sw128(vb + kk * 2048, kHalf, 1024), idesc_pv,
                  (j > 0 || kk > 0) ? 1u : 0u);
        }
      };
      ok = mbar_wait(&bar.q_full, 0) && mbar_wait(&bar.k_full[0], 0);
      if (ok) {
        tc_fence_after();
        qk(0, 0);
        qk(1, 0);
        umma_commit(&bar.k_empty[0]);
      }
      for (int j = 0; j < nkv && ok; ++j) {
        const int vs = j % kVStages;
        const bool more = j + 1 < nkv;
        // tile A: PV_A(j), then S_A(j+1) (after PV_A(j) in issue order, which
        // the tensor core preserves, so P_A(j) is consumed before it is overwritten)
        ok = mbar_wait(&bar.p_full[0], j & 1) && mbar_wait(&bar.v_full[vs], (j / kVStages) & 1);
        if (ok && more) ok = mbar_wait(&bar.k_full[(j + 1) % kKStages], ((j + 1) / kKStages) & 1);
        if (!ok) break;
        tc_fence_after();
        pv(0, j);
        if (!more) umma_commit(&bar.o_final[0]);
        if (more) qk(0, j + 1);
        // tile B
        ok = mbar_wait(&bar.p_full[1], j & 1);
        if (!ok) break;
        tc_fence_after();
        pv(1, j);
        umma_commit(&bar.v_empty[vs]);
        if (!more) umma_commit(&bar.o_final[1]);
        if (more) {
          qk(1, j + 1);
          umma_commit(&bar.k_empty[(j + 1) % kKStages]);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int t = warp >> 2;                  // Q tile (A = 0, B = 1)
    const int r = threadIdx.x & (kBM - 1);    // row of the tile == TMEM lane
    const int tq = tq0 + t * a.tt + r / a.g;  // token within the sequence
    const int qpos = p0 + tq;
    const int qpos_min = p0 + tq0 + t * a.tt;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_base + TM_S + t * kBM;
    const uint32_t tO = tmem + lane_base + TM_O + t * kBM;
    float m_run = -INFINITY, l_run = 0.f;
    float sv[kBN];
    for (int j = 0; j < nkv; ++j) {
      ok = mbar_wait(&bar.s_full[t], j & 1);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      tmem_ld128(tS, sv);
      const int kbase = j * kBN;
      if (kbase + kBN - 1 > qpos_min) {
#pragma unroll
        for (int i = 0; i < kBN; ++i) {
          if (kbase + i > qpos) sv[i] = -INFINITY;
        }
      }
      // 8 independent max / sum chains
      float mx8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mx8[k] = sv[k];
#pragma unroll
      for (int i = 8; i < kBN - 8; i += 16) {
#pragma unroll
        for (int k = 0; k < 8; ++k) mx8[k] = fmax3(mx8[k], sv[i + k], sv[i + 8 + k]);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) mx8[k] = fmaxf(mx8[k], sv[kBN - 8 + k]);
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      // scores are raw q.k; the softmax scale (and log2 e) folds into one FFMA
      const float m_new = fmaxf(m_run, mx * a.scale_log2);
      const bool need = j > 0 && (m_new - m_run > kRescaleThreshold);
      const float m_use = (j == 0 || need) ? m_new : m_run;
      const float corr = j == 0 ? 0.f : fast_exp2(m_run - m_use);
      // exponentials, row sum and P (bf16 pairs) in two 64-key halves so P
      // of the first half is in TMEM before the second half is computed
      // (scale and max subtraction, and the 8 running sums, on packed fp32
      // pairs: the same roundings as the scalar FFMA / FADD, half the issue)
      uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};
      const uint64_t sc2 = f32x2(a.scale_log2, a.scale_log2), nm2 = f32x2(-m_use, -m_use);
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t pw[32];
#pragma unroll
        for (int i = 0; i < kBN / 2; i += 8) {
#pragma unroll
          for (int k = 0; k < 8; k += 2) {
            float x0, x1;
            f32x2_split(f32x2_fma(f32x2(sv[hf * 64 + i + k], sv[hf * 64 + i + k + 1]), sc2, nm2),
                        x0, x1);
            const float e0 = ((kEmuMask >> k) & 1u) ? poly_exp2(x0) : fast_exp2(x0);
            const float e1 = ((kEmuMask >> (k + 1)) & 1u) ? poly_exp2(x1) : fast_exp2(x1);
            sum2[k / 2] = f32x2_add(sum2[k / 2], f32x2(e0, e1));
            pw[(i + k) / 2] = pack_bf16(e0, e1);
          }
        }
        tmem_st32u_nowait(tS + hf * 32, pw);
      }
      float sum8[8];
#pragma unroll
      for (int k = 0; k < 8; k += 2) f32x2_split(sum2[k / 2], sum8[k], sum8[k + 1]);
      const float sum = ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) +
                        ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
      l_run = l_run * corr + sum;
      m_run = m_use;
      // PV_t(j-1) completed before S_t(j) (commit after QK_t(j) covers it),
      // so O may be rescaled here without another wait.
      if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
        for (int c = 0; c < kD / 32; ++c) {
          float o[32];
          tmem_ld32(tO + c * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= corr;
          tmem_st32(tO + c * 32, o);
        }
        tmem_st_wait();
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bar.p_full[t]);
    }
    // ---- epilogue: O / l -> bf16 rows of the packed output
    if (ok) ok = mbar_wait(&bar.o_final[t], 0);
    if (__all_sync(0xffffffffu, ok)) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      const bool valid = tq < n && q0 + tq < a.num_tokens;
      __nv_bfloat16 *orow =
          a.out + ((size_t)(q0 + tq) * a.Hq + (size_t)h * a.g + (r % a.g)) * kD;
#pragma unroll 1
      for (int c = 0; c < kD / 32; ++c) {
        float o[32];
        tmem_ld32(tO + c * 32, o);
        if (valid) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            w.x = pack_bf16(o[i] * inv, o[i + 1] * inv);
            w.y = pack_bf16(o[i + 2] * inv, o[i + 3] * inv);
            w.z = pack_bf16(o[i + 4] * inv, o[i + 5] * inv);
            w.w = pack_bf16(o[i + 6] * inv, o[i + 7] * inv);
            *reinterpret_cast<uint4 *>(orow + c * 32 + i) = w;
          }
        }
      }
    } else {
      ok = false;
    }
  }
  if (!ok) atomicExch(a.err, 1);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kWarpMma) tmem_dealloc(tmem, 512);
}

// 11 warps: a sub-partition holds 3 of them in its 16K registers -> <= 168 each.
__global__ void __launch_bounds__(kThreads, 1)
prefill_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
               const __grid_constant__ CUtensorMap tmv, PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  // longest tile pairs first
  prefill_body(&tmq, &tmk, &tmv, a, blockIdx.z, blockIdx.y, gridDim.x - 1 - blockIdx.x,
               smem_raw);
}

// Mixed step (chunked prefill): one launch runs the decode rows and the
// prompt chunks. CTAs [0, n_dec) are decode CTAs: kMixedDecodeWarps warps
// each run the split-KV decode warp loop (work items pulled from the
// workspace's queue, as in decode_chunk_kernel); the other warps leave. The
// remaining CTAs are prefill tile pairs, numbered pair-fastest, then kv head,
// then sequence (the 3-D grid of prefill_kernel, flattened). One CTA fits an
// SM (shared memory), so decode CTAs stream K/V on their SMs while prefill
// CTAs keep the tensor cores busy on the others.
constexpr int kMixedDecodeWarps = 8;
static_assert(dk::smem_bytes(kMixedDecodeWarps) <= kSmemBytes, "decode CTAs fit the smem");

__global__ void __launch_bounds__(kThreads, 1)
attention_mixed_kernel(const __grid_constant__ CUtensorMap tmq,
                       const __grid_constant__ CUtensorMap tmk,
                       const __grid_constant__ CUtensorMap tmv, PrefillArgs pa,
                       dk::DecodeArgs da, int n_dec, int mpairs, int n_pre_ctas,
                       int num_seqs) {
  extern __shared__ uint8_t smem_raw[];
  if (static_cast<int>(blockIdx.x) >= n_dec + n_pre_ctas) {
    // rows past cu_seqlens_q[num_seqs] (padding) -> 0
    const int64_t row_elems = (int64_t)pa.Hq * kD;
    const int64_t start = (int64_t)__ldg(pa.cu - da.B + num_seqs) * row_elems;
    const int64_t end = (int64_t)pa.num_tokens * row_elems;
    const int64_t tail = static_cast<int>(blockIdx.x) - n_dec - n_pre_ctas;
    const int64_t n_tail = gridDim.x - n_dec - n_pre_ctas;
    uint4 *o = reinterpret_cast<uint4 *>(pa.out);
    for (int64_t i = start / 8 + tail * blockDim.x + threadIdx.x; i < end / 8;
         i += n_tail * blockDim.x) {
      o[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    return;
  }
  if (static_cast<int>(blockIdx.x) < n_dec) {
    const int warp = threadIdx.x >> 5;
    if (warp >= kMixedDecodeWarps) return;   // decode CTAs use no block-wide barrier
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    dk::decode_chunk_body<kMixedDecodeWarps>(&tmk, &tmv, da, smem, warp, threadIdx.x & 31);
    return;
  }
  const int idx = static_cast<int>(blockIdx.x) - n_dec;
  const int x = idx % mpairs, rest = idx / mpairs;
  prefill_body(&tmq, &tmk, &tmv, pa, rest / pa.Hkv, rest % pa.Hkv, mpairs - 1 - x, smem_raw);
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
  CUtensorMap tmq, tmk, tmv;
  // Q: dims (D, Hq, tokens); one box = the g heads of tt tokens, 64 dims
  int rc = encode_tmap_3d(&tmq, q, kD, num_q_heads, num_tokens, (uint64_t)kD * 2,
                          (uint64_t)num_q_heads * kD * 2, 64, g, tt, true);
  if (rc) return rc;
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
  const int64_t mpairs = (maxq + 2 * tt - 1) / (2 * tt);
  if (num_seqs > 0 && mpairs > 0) {
    if (mpairs > INT32_MAX || num_kv_heads > 65535 || num_seqs > 65535) {
      return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_prefill: grid too large");
    }
    cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)kSmemBytes);
    dim3 grid((unsigned)mpairs, num_kv_heads, num_seqs);
    prefill_kernel<<<grid, kThreads, kSmemBytes, stream>>>(tmq, tmk, tmv, a);
    rc = check_launch("vj_paged_prefill");
    if (rc) return rc;
  }
  prefill_zero_tail_kernel<<<num_sms() * 2, 256, 0, stream>>>(
      static_cast<__nv_bfloat16 *>(out), cu_seqlens_q, num_seqs, num_tokens, num_q_heads * kD);
  return check_launch("vj_paged_prefill(zero tail)");
}

extern "C" size_t vj_paged_attention_mixed_workspace_size(int32_t num_decode,
                                                          int32_t num_q_heads, int32_t head_dim,
                                                          int32_t max_chunks) {
  if (num_decode < 0 || num_q_heads <= 0 || head_dim != vj::kD) return 0;
  if (max_chunks <= 0) max_chunks = 4096 + num_decode;
  return vj::dk::workspace_bytes(num_decode, num_q_heads, max_chunks);
}

extern "C" vj_status vj_paged_attention_mixed(
    const void *q, const void *k_cache, const void *v_cache, const int32_t *block_tables,
    const int32_t *cu_seqlens_q, const int32_t *context_lens, void *out, int64_t num_tokens,
    int32_t num_seqs, int32_t num_decode, int32_t num_q_heads, int32_t num_kv_heads,
    int32_t head_dim, int64_t num_blocks, int32_t block_size, int32_t bt_width,
    int32_t bt_stride, int64_t stride_block, int64_t stride_token, int64_t stride_head,
    int32_t max_seqlen_q, float scale, int32_t max_chunks, int32_t plan, void *workspace,
    size_t workspace_bytes, int32_t *error_flag, cudaStream_t stream) {
  using namespace vj;
  if (num_tokens < 0 || num_seqs < 0 || num_decode < 0 || num_decode > num_seqs ||
      num_q_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 || bt_width < 0 ||
      bt_stride < bt_width) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_paged_attention_mixed: bad sizes");
  }
  if (num_q_heads % num_kv_heads != 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_paged_attention_mixed: Number of Q heads must be divisible by number "
                     "of KV heads");
  }
  const int g = num_q_heads / num_kv_heads;
  if (head_dim != kD) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_attention_mixed: head_dim must be 128");
  }
  if (g > 8 || kBM % g != 0 || num_kv_heads > 255) {
    return set_error(VJ_ERR_UNSUPPORTED,
                     "vj_paged_attention_mixed: query heads per KV head must be <= 8 and divide "
                     "128; at most 255 KV heads");
  }
  if (block_size <= 0 || block_size % kPageTok != 0 ||
      stride_block != (int64_t)block_size * stride_token) {
    return set_error(VJ_ERR_UNSUPPORTED,
                     "vj_paged_attention_mixed: block_size must be a multiple of 16 with evenly "
                     "strided tokens");
  }
  if (num_blocks * block_size > (int64_t)INT32_MAX || num_tokens > (int64_t)INT32_MAX) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_attention_mixed: sizes beyond 2^31");
  }
  if (num_tokens == 0 || num_seqs == 0) return VJ_OK;
  if (!q || !k_cache || !v_cache || !block_tables || !cu_seqlens_q || !context_lens || !out ||
      !error_flag) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_paged_attention_mixed: null pointer");
  }
  if (max_chunks <= 0) max_chunks = 4096 + num_decode;
  if (num_decode > 0) {
    if (max_chunks <= num_decode || max_chunks >= (1 << 23)) {
      return set_error(VJ_ERR_INVALID_ARGUMENT,
                       "vj_paged_attention_mixed: max_chunks must exceed num_decode, below 2^23");
    }
    const size_t need = dk::workspace_bytes(num_decode, num_q_heads, max_chunks);
    if (!workspace || workspace_bytes < need ||
        reinterpret_cast<uintptr_t>(workspace) % 16 != 0) {
      return set_error(VJ_ERR_WORKSPACE, "vj_paged_attention_mixed: workspace needs " +
                                             std::to_string(need) + " bytes, 16-byte aligned");
    }
  }
  const int tt = kBM / g;
  CUtensorMap tmq, tmk, tmv;
  int rc = encode_tmap_3d(&tmq, q, kD, num_q_heads, num_tokens, (uint64_t)kD * 2,
                          (uint64_t)num_q_heads * kD * 2, 64, g, tt, true);
  if (rc) return rc;
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
  // prompt chunks: sequences [num_decode, num_seqs)
  const int n_pre = num_seqs - num_decode;
  PrefillArgs pa;
  pa.out = static_cast<__nv_bfloat16 *>(out);
  pa.bt = block_tables + (size_t)num_decode * bt_stride;
  pa.cu = cu_seqlens_q + num_decode;
  pa.ctx_lens = context_lens + num_decode;
  pa.Hq = num_q_heads; pa.Hkv = num_kv_heads; pa.g = g; pa.tt = tt;
  pa.bt_stride = bt_stride;
  pa.pages_per_block = block_size / kPageTok;
  pa.max_pages = bt_width * pa.pages_per_block;
  pa.block_size = block_size;
  pa.num_blocks = (int)num_blocks;
  pa.head_major = head_major ? 1 : 0;
  pa.num_tokens = (int)num_tokens;
  pa.scale_log2 = scale * kLog2e;
  pa.err = error_flag;
  // decode rows: sequences [0, num_decode), q row b = sequence b
  dk::DecodeArgs da{};
  da.q = static_cast<const __nv_bfloat16 *>(q);
  da.out = static_cast<__nv_bfloat16 *>(out);
  da.bt = block_tables;
  da.lens = context_lens;
  da.B = num_decode; da.Hq = num_q_heads; da.Hkv = num_kv_heads; da.g = g;
  da.bt_stride = bt_stride;
  da.pages_per_block = block_size / kPageTok;
  da.max_pages = bt_width * da.pages_per_block;
  da.block_size = block_size;
  da.num_blocks = (int)num_blocks;
  da.head_major = head_major ? 1 : 0;
  da.scale_log2 = scale * kLog2e;
  // decode CTAs: half the SMs when prompt chunks share the launch, else all
  const int n_dec = num_decode == 0 ? 0 : (n_pre > 0 ? std::max(1, num_sms() / 2) : num_sms());
  if (num_decode > 0) {
    da.ws = dk::carve(workspace, num_decode, num_q_heads, max_chunks);
    if (plan) {
      dk::decode_plan_kernel<<<1, 1024, 0, stream>>>(context_lens, num_decode, num_kv_heads,
                                                     max_chunks, n_dec * kMixedDecodeWarps,
                                                     da.max_pages, da.ws);
      rc = check_launch("vj_paged_attention_mixed(plan)");
      if (rc) return rc;
    }
  }
  const int64_t maxq = max_seqlen_q > 0 ? max_seqlen_q : num_tokens;
  const int64_t mpairs = n_pre > 0 ? std::max<int64_t>(1, (maxq + 2 * tt - 1) / (2 * tt)) : 1;
  const int64_t n_pre_ctas = n_pre > 0 ? mpairs * num_kv_heads * n_pre : 0;
  constexpr int kTailCtas = 8;   // zero the rows past cu_seqlens_q[num_seqs]
  const int64_t grid = n_dec + n_pre_ctas + kTailCtas;
  if (grid > INT32_MAX) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_attention_mixed: grid too large");
  }
  cudaFuncSetAttribute(attention_mixed_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)kSmemBytes);
  attention_mixed_kernel<<<(unsigned)grid, kThreads, kSmemBytes, stream>>>(
      tmq, tmk, tmv, pa, da, n_dec, (int)mpairs, (int)n_pre_ctas, num_seqs);
  rc = check_launch("vj_paged_attention_mixed");
  if (rc) return rc;
  if (num_decode > 0) {
    const int warps = num_decode * num_q_heads;
    dk::decode_combine_kernel<<<(warps + 7) / 8, 256, 0, stream>>>(da);
    rc = check_launch("vj_paged_attention_mixed(combine)");
  }
  return rc;
}
