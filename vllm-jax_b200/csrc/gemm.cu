// Decode-step projections on tcgen05 with their elementwise successors fused
// into the epilogue:
//
//   vj_qkv_gemm_kv_store  q|k|v = x Wqkv^T, then in the epilogue K3's q/k
//                         RMSNorm + interleaved-pair RoPE + q scaling + KV-slot
//                         store (kv_row.cuh): the projected q/k/v rows never
//                         reach HBM, and K3's launch disappears.
//                         Replaces vllm/model/qwen3.py:286-296 (qkv projection,
//                         q_norm/k_norm, apply_rope) and :105-111 (_update_kv_cache).
//   vj_decode_gemm        out = x W^T (PLAIN), or SwiGLU: out = silu(x Wg^T) *
//                         (x Wu^T) (qwen3.py:337-341), so the [T, 2I] gate/up
//                         output and the separate SiLU-mul pass disappear.
//
// Shape: decode batches (T up to a few hundred rows) against weights of
// 10^7-10^8 elements, so a launch is a weight stream: every weight byte is read
// once from HBM; x (T x K bf16, at most a few MB) stays in L2.
//
// Operand roles ("swap AB"): the MMA's M side is 128 weight rows (output
// features), its N side the call's tokens, padded to a multiple of 16 (at most
// 128 per m tile), so a batch of 8 tokens moves and multiplies 16 token rows,
// not 128. D^T[feature, token] accumulates in TMEM, one feature per lane.
//
// Tiling: a work unit is one 128-row weight tile (n) x one tile of <= 128
// tokens (m) x one contiguous range of the K blocks (split). Splits are chosen
// on the host so that the units fill the SMs in whole waves; a persistent CTA
// per SM walks units u = blockIdx.x, +gridDim.x, ... Consecutive units share
// their weight tile (different m), so a weight tile comes from HBM once.
//
// CTA = 6 warps:
//   warp 0      TMA producer: per K block two 64x64 weight boxes and one x box
//               (n_pad tokens x 64), 128-byte swizzle, into a ring of up to 12
//               stages in 192 KB (160 KB with a cluster reduction); packed
//               weights come as one 16 KB bulk copy per stage instead
//   warp 1      TMEM owner + MMA issuer: tcgen05.mma kind::f16, M = 128,
//               N = n_pad, K = 16, both operands K-major in shared memory; the
//               256 TMEM columns hold 2 (n_pad > 64), 4 (> 32) or 8
//               accumulators, so the MMAs run that many units ahead of the
//               epilogue
//   warps 2-5   epilogue: lane f holds feature f of every token; with a K
//               split the fp32 partials go through the workspace (the last of
//               a tile's splits to arrive -- atomicInc ticket, threadfence-
//               reduction pattern, no CTA ever waits for another -- sums them
//               in split order, so results do not depend on timing); on
//               request (2-8 splits, <= 64 tokens) the splits of a tile are
//               one thread-block cluster instead and sum their partials in
//               rank order through distributed shared memory (remote mbarrier
//               arrivals, bounded waits), each rank finishing 1/C of the
//               tokens; the bf16
//               tile is transposed into a [token][feature] shared-memory tile,
//               from which the mode's row pass stores (PLAIN), applies SiLU-mul
//               (SWIGLU) or runs K3's 8-lane row code (KV)
// Every mbarrier wait is bounded (2 s); a timeout sets the caller's error word.
#include "../../include/vjattn.h"
#include "vj_common.cuh"
#include "kv_row.cuh"

#include <algorithm>
#include <string>

namespace vj {
namespace {

constexpr int kBM = 128;           // tokens per m tile (MMA N at most)
constexpr int kBN = 128;           // weight rows per tile (MMA M)
constexpr int kBK = 64;            // K elements per stage (one 128-byte swizzle row)
constexpr int kMaxStages = 12;
constexpr int kTileBytes = kBN * kBK * 2;      // 16 KB: the weight tile of a K block
// Shared memory: the stage ring ([weight tile][x box] per stage), then the
// bf16 staging tile; with a cluster reduction the ring gives up 32 KB to the
// fp32 partial buffer: [ring 160 KB][staging][red] instead of [ring 192 KB][staging].
constexpr int kRingBytes = 192 * 1024;
constexpr int kRingBytesCluster = 160 * 1024;
constexpr int kGemmThreads = 192;
constexpr int kEpiThreads = 128;
constexpr int kStagingBytes = kBM * 256;       // one bf16 [token][feature] tile
constexpr int kRedBytes = 64 * kBN * 4;        // fp32 [token][feature] partial, <= 64 tokens
constexpr int kMaxCluster = 8;
constexpr int kMaxSplits = 32;
// The workspace starts with a fixed ticket area (one word per output tile of
// a split-K call), the same for every shape, so that calls of different shapes
// sharing one workspace never write partials over another call's tickets.
constexpr int kMaxTicketTiles = 16384;
constexpr size_t kTicketBytes = kMaxTicketTiles * sizeof(unsigned);

enum { kModePlain = 0, kModeSwiglu = 1, kModeKv = 2 };

struct GemmArgs {
  int rows;                 // T
  int kblocks;              // K / 64
  int m_tiles, n_tiles, splits, units;
  int n_pad;                // tokens per m tile rounded up to 16 (MMA N), <= 128
  int cluster;              // > 1: the splits of a tile are one thread-block cluster
                            // and reduce through distributed shared memory
  int nbuf;                 // TMEM accumulators (256 / nbuf columns each)
  int mode;
  int stages;               // ring depth
  int stage_bytes;          // 16 KB of weights + n_pad x 128 B of x
  int inter;                // SwiGLU: intermediate size I (gate rows [0,I), up rows [I,2I))
  const uint8_t *wtiles;    // weights packed by vj_pack_weight_tiles (or NULL: tensor map)
  __nv_bfloat16 *out;       // PLAIN [T, N] / SwiGLU [T, I], row stride ldo
  int64_t ldo;
  float *partials;          // [tiles][splits][128 tokens][128 features] fp32 (splits > 1)
  unsigned int *tickets;    // [tiles]
  int *error;
};

struct Smem {
  uint64_t full[kMaxStages], empty[kMaxStages];
  uint64_t acc_full[8], acc_empty[8], drain;
  uint64_t red_ready, red_free;   // cluster reduction: partials published / consumed
  uint32_t tmem_base;
  int ticket;
};
constexpr int kOffRed = kRingBytesCluster + kStagingBytes;
constexpr int kOffBars = kRingBytes + kStagingBytes;
static_assert(kOffRed + kRedBytes == kOffBars, "shared-memory layout");
constexpr int kSmemBytes = kOffBars + static_cast<int>(sizeof(Smem)) + 1024;  // + alignment slack

// Barrier among `count` threads that also ANDs their predicates, so that a
// wait that ran out for some epilogue threads stops all of them together.
VJ_DEV bool bar_and(uint32_t id, uint32_t count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

VJ_DEV void flag_error(int *error) {
  if (error) atomicExch(error, 1);
}

// Distributed shared memory (thread-block cluster) helpers.
VJ_DEV uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Arrive (release, cluster scope) on an mbarrier of a CTA in this cluster.
VJ_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
VJ_DEV bool mbar_try_wait_acq_cluster(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded (2 s) wait with cluster-scope acquire: peers' writes published
// before their arrivals are visible afterwards.
VJ_DEV bool mbar_wait_cluster(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait_acq_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_acq_cluster(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}
VJ_DEV float ld_dsmem_f32(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}
// All threads of all CTAs of the cluster (a lone CTA is a cluster of one).
VJ_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

// Unit u -> (m tile, n tile, split); m fastest so that neighbouring CTAs
// stream the same weight tile.
VJ_DEV void unit_coords(const GemmArgs &g, int u, int &mt, int &nt, int &sp) {
  mt = u % g.m_tiles;
  const int r = u / g.m_tiles;
  sp = r % g.splits;
  nt = r / g.splits;
}
// The j-th unit of this CTA. Without a cluster: units blockIdx.x + j *
// gridDim.x; with clusters of C CTAs: tile (cluster + j * clusters), split =
// the CTA's rank in its cluster. False when the CTA has no j-th unit.
VJ_DEV bool unit_at(const GemmArgs &g, int j, int &mt, int &nt, int &sp) {
  if (g.cluster <= 1) {
    const int u = blockIdx.x + j * gridDim.x;
    if (u >= g.units) return false;
    unit_coords(g, u, mt, nt, sp);
    return true;
  }
  const int C = g.cluster;
  const int tile = static_cast<int>(blockIdx.x) / C + j * (static_cast<int>(gridDim.x) / C);
  if (tile >= g.m_tiles * g.n_tiles) return false;
  mt = tile % g.m_tiles;
  nt = tile / g.m_tiles;
  sp = static_cast<int>(blockIdx.x) % C;
  return true;
}
VJ_DEV int split_begin(const GemmArgs &g, int sp) {
  return static_cast<int>((static_cast<int64_t>(sp) * g.kblocks) / g.splits);
}

// Weight rows of n tile nt: two 64-row boxes. PLAIN/KV: rows [128 nt, +128);
// SwiGLU: gate rows [64 nt, +64) then up rows [I + 64 nt, +64), so the tile's
// features 0-63 are gate and 64-127 up for the same 64 outputs.
VJ_DEV void weight_rows(const GemmArgs &g, int nt, int &r0, int &r1) {
  if (g.mode == kModeSwiglu) {
    r0 = 64 * nt;
    r1 = g.inter + 64 * nt;
  } else {
    r0 = kBN * nt;
    r1 = kBN * nt + 64;
  }
}

// SiLU-mul of one output element, the same arithmetic as vj_silu_mul:
// bf16(bf16(silu(g)) * u) with g, u the bf16-rounded projections.
VJ_DEV float swiglu(float gate, float up) {
  const float g = round_bf16(gate);
  const float u = round_bf16(up);
  const float s = round_bf16(g / (1.f + expf(-g)));
  return s * u;
}

// Byte offset of (token row t, 16-byte chunk c) in the staging tile: chunk c
// of row t sits at chunk c ^ (t & 15), so that a warp writing 32 features of
// one token and 8 lanes reading 8 chunks of one row both hit distinct banks.
VJ_DEV uint32_t stg_off(int t, int c) {
  return static_cast<uint32_t>(t) * 256u + (static_cast<uint32_t>(c ^ (t & 15)) << 4);
}

__global__ void __launch_bounds__(kGemmThreads, 1)
decode_gemm_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
                   const GemmArgs g, const KvArgs kv) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  Smem &sb = *reinterpret_cast<Smem *>(smem + kOffBars);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < g.stages; ++i) {
      mbar_init(&sb.full[i], 1);
      mbar_init(&sb.empty[i], 1);
    }
    for (int i = 0; i < g.nbuf; ++i) {
      mbar_init(&sb.acc_full[i], 1);
      mbar_init(&sb.acc_empty[i], kEpiThreads);
    }
    mbar_init(&sb.drain, 1);
    mbar_init(&sb.red_ready, g.cluster);
    mbar_init(&sb.red_free, g.cluster);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&sb.tmem_base, 256);
  tc_fence_before();
  __syncthreads();
  // every CTA of the cluster has initialised its barriers before any remote
  // arrival
  if (g.cluster > 1) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = sb.tmem_base;
  const uint32_t S = static_cast<uint32_t>(g.stages);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmx);
      if (g.wtiles == nullptr) tma_prefetch_desc(&tmw);
      uint32_t it = 0;
      bool ok = true;
      int mt, nt, sp;
      for (int j = 0; ok && unit_at(g, j, mt, nt, sp); ++j) {
        int wr0, wr1;
        weight_rows(g, nt, wr0, wr1);
        const int kb1 = split_begin(g, sp + 1);
        for (int kb = split_begin(g, sp); kb < kb1; ++kb, ++it) {
          const int st = static_cast<int>(it % S);
          if (it >= S && !mbar_wait(&sb.empty[st], ((it / S) - 1) & 1)) {
            ok = false;
            break;
          }
          uint8_t *dst = smem + st * g.stage_bytes;
          mbar_arrive_expect_tx(&sb.full[st], g.stage_bytes);
          if (g.wtiles != nullptr) {
            // packed weights: the stage's 16 KB tile is one contiguous block,
            // already in the swizzled order, moved by one bulk copy
            bulk_g2s(dst, g.wtiles + (static_cast<size_t>(nt) * g.kblocks + kb) * kTileBytes,
                     kTileBytes, &sb.full[st]);
          } else {
            tma_load_3d(dst, &tmw, &sb.full[st], kb * kBK, wr0, 0);
            tma_load_3d(dst + kTileBytes / 2, &tmw, &sb.full[st], kb * kBK, wr1, 0);
          }
          tma_load_3d(dst + kTileBytes, &tmx, &sb.full[st], kb * kBK, mt * kBM, 0);
        }
      }
      if (!ok) {
        flag_error(g.error);
        // copies in flight must land before the CTA exits
        for (uint32_t j = it > S ? it - S : 0; j < it; ++j) {
          mbar_wait(&sb.full[j % S], (j / S) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(kBN, g.n_pad, false);
      const uint32_t s0 = smem_u32(smem);
      uint32_t it = 0;
      bool ok = true;
      int mt, nt, sp;
      for (int j = 0; ok && unit_at(g, j, mt, nt, sp); ++j) {
        const int buf = j % g.nbuf;
        if (j >= g.nbuf && !mbar_wait(&sb.acc_empty[buf], ((j / g.nbuf) - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * (256 / g.nbuf);
        const int kb0 = split_begin(g, sp), kb1 = split_begin(g, sp + 1);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int st = static_cast<int>(it % S);
          if (!mbar_wait(&sb.full[st], (it / S) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t wa = s0 + st * g.stage_bytes, xa = wa + kTileBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            umma_ss(d, umma_desc_sw128(wa + kk * 32, 16, 1024),
                    umma_desc_sw128(xa + kk * 32, 16, 1024), idesc,
                    (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&sb.empty[st]);
        }
        if (ok) umma_commit(&sb.acc_full[buf]);
      }
      if (!ok) flag_error(g.error);
      // every issued MMA completes before TMEM is released
      umma_commit(&sb.drain);
      mbar_wait(&sb.drain, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int et = threadIdx.x - 64;                 // 0..127
    const int quarter = warp & 3;                    // TMEM lane quarter of this warp
    const int f = quarter * 32 + lane;               // feature (weight row) of the tile
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    uint8_t *staging = smem + (g.cluster > 1 ? kRingBytesCluster : kRingBytes);
    // K3 state (KV mode): 16 groups of 8 lanes
    const int grp = et >> 3, l8 = et & 7;
    const unsigned grp_mask = 0xffu << (8 * (grp & 3));
    RowSlice qw, kw;
    if (g.mode == kModeKv) load_weights(kv, l8, qw, kw);
    const int nchunks = (g.n_pad + 31) / 32;
    float *red = reinterpret_cast<float *>(smem + kOffRed);
    uint32_t red_peer[kMaxCluster];
    for (int q = 0; q < kMaxCluster; ++q) {
      red_peer[q] = q < g.cluster ? mapa_shared(smem_u32(red), q) : 0u;
    }
    int mt, nt, sp;
    for (int j = 0; unit_at(g, j, mt, nt, sp); ++j) {
      const int buf = j % g.nbuf;
      if (!bar_and(1, kEpiThreads, mbar_wait(&sb.acc_full[buf], (j / g.nbuf) & 1))) {
        if (et == 0) flag_error(g.error);
        break;
      }
      tc_fence_after();
      const uint32_t tacc = tmem + lane_addr + buf * (256 / g.nbuf);
      const int nlive = min(kBM, g.rows - mt * kBM);     // tokens of this m tile
      const int tile = nt * g.m_tiles + mt;
      const float *part = g.partials + static_cast<size_t>(tile) * g.splits * (kBM * kBN) + f;
      int tb = 0, te = nlive;   // the tokens of the tile this CTA finishes
      if (g.cluster > 1) {
        // K splits of this tile = the CTAs of this cluster. Each publishes its
        // fp32 partial [token][feature] in its own shared memory, then
        // finishes a 1/C share of the tokens, summing the C partials in rank
        // order through distributed shared memory.
        const int C = g.cluster;
        const int per = (nlive + C - 1) / C;
        tb = min(nlive, sp * per);
        te = min(nlive, tb + per);
        // the peers have read this buffer's previous tile
        if (j > 0 && !bar_and(1, kEpiThreads, mbar_wait_cluster(&sb.red_free, (j - 1) & 1))) {
          if (et == 0) flag_error(g.error);
          break;
        }
#pragma unroll 1
        for (int c = 0; c < nchunks; ++c) {
          float v[32];
          tmem_ld32(tacc + c * 32, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (c * 32 + i < nlive) red[(c * 32 + i) * kBN + f] = v[i];
          }
        }
        tc_fence_before();
        mbar_arrive(&sb.acc_empty[buf]);
        named_bar_sync(1, kEpiThreads);
        if (et == 0) {
          for (int q = 0; q < C; ++q) mbar_arrive_cluster(mapa_shared(smem_u32(&sb.red_ready), q));
        }
        if (!bar_and(1, kEpiThreads, mbar_wait_cluster(&sb.red_ready, j & 1))) {
          if (et == 0) flag_error(g.error);
          break;
        }
        for (int t = tb; t < te; ++t) {
          float pv[kMaxCluster];
#pragma unroll
          for (int q = 0; q < kMaxCluster; ++q) {
            if (q < C) pv[q] = ld_dsmem_f32(red_peer[q] + static_cast<uint32_t>(t * kBN + f) * 4u);
          }
          float acc = pv[0];
#pragma unroll
          for (int q = 1; q < kMaxCluster; ++q) {
            if (q < C) acc += pv[q];
          }
          *reinterpret_cast<__nv_bfloat16 *>(staging + stg_off(t, f >> 3) + (f & 7) * 2) =
              __float2bfloat16_rn(acc);
        }
        named_bar_sync(1, kEpiThreads);   // this CTA's reads of every peer are done
        if (et == 0) {
          for (int q = 0; q < C; ++q) mbar_arrive_cluster(mapa_shared(smem_u32(&sb.red_free), q));
        }
      } else {
      if (g.splits > 1) {
        // this split's partial tile to the workspace ([token][feature]:
        // coalesced); tcgen05.ld is warp-collective, so every lane loads
#pragma unroll 1
        for (int c = 0; c < nchunks; ++c) {
          float v[32];
          tmem_ld32(tacc + c * 32, v);
          float *mine = g.partials + (static_cast<size_t>(tile) * g.splits + sp) * (kBM * kBN) +
                        static_cast<size_t>(c * 32) * kBN + f;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (c * 32 + i < nlive) __stcg(mine + i * kBN, v[i]);
          }
        }
        __threadfence();
        named_bar_sync(1, kEpiThreads);
        if (et == 0) sb.ticket = static_cast<int>(atomicInc(g.tickets + tile, g.splits - 1));
        named_bar_sync(1, kEpiThreads);
        if (sb.ticket != g.splits - 1) {   // another split finishes this tile
          tc_fence_before();
          mbar_arrive(&sb.acc_empty[buf]);
          continue;
        }
        __threadfence();
      }
      // feature f of tokens [32c, 32c+32): this split's accumulator plus,
      // with a K split, every split's partial in split order; each split's
      // 16 values are loaded together, the next split's while the current
      // ones are added. The bf16 results go to the staging tile.
#pragma unroll 1
      for (int c = 0; c < nchunks; ++c) {
        float v[32];
        tmem_ld32(tacc + c * 32, v);
        if (g.splits > 1) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int t0 = c * 32 + h * 16;
            if (t0 >= nlive) break;
            const float *pc = part + static_cast<size_t>(t0) * kBN;
            float acc[16], cur[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              cur[i] = (sp == 0 || t0 + i >= nlive) ? v[h * 16 + i] : __ldcg(pc + i * kBN);
            }
#pragma unroll 1
            for (int q = 0; q < g.splits; ++q) {
              float nxt[16];
              const int qn = q + 1;
              if (qn < g.splits) {
                const float *pn = pc + static_cast<size_t>(qn) * (kBM * kBN);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  nxt[i] = (qn == sp || t0 + i >= nlive) ? v[h * 16 + i] : __ldcg(pn + i * kBN);
                }
              }
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                acc[i] = q == 0 ? cur[i] : acc[i] + cur[i];
                cur[i] = nxt[i];
              }
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) v[h * 16 + i] = acc[i];
          }
        }
        // transpose into staging[token][feature] (bf16)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int t = c * 32 + i;
          if (t < nlive) {
            *reinterpret_cast<__nv_bfloat16 *>(staging + stg_off(t, f >> 3) + (f & 7) * 2) =
                __float2bfloat16_rn(v[i]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&sb.acc_empty[buf]);
      named_bar_sync(1, kEpiThreads);
      }

      const int64_t t_base = static_cast<int64_t>(mt) * kBM;
      if (g.mode == kModePlain) {
        // 16 chunks of 16 bytes per token row, 8 rows per pass
        const int c = et & 15;
        for (int t = tb + (et >> 4); t < te; t += kEpiThreads / 16) {
          const uint4 w = *reinterpret_cast<const uint4 *>(staging + stg_off(t, c));
          *reinterpret_cast<uint4 *>(g.out + (t_base + t) * g.ldo +
                                     static_cast<int64_t>(nt) * kBN + c * 8) = w;
        }
      } else if (g.mode == kModeSwiglu) {
        // 8 outputs (a gate chunk and its up chunk) per thread, 16 rows per pass
        const int c = et & 7;
        for (int t = tb + (et >> 3); t < te; t += kEpiThreads / 8) {
          const uint4 gw = *reinterpret_cast<const uint4 *>(staging + stg_off(t, c));
          const uint4 uw = *reinterpret_cast<const uint4 *>(staging + stg_off(t, 8 + c));
          const uint32_t ga[4] = {gw.x, gw.y, gw.z, gw.w}, ua[4] = {uw.x, uw.y, uw.z, uw.w};
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            o[i] = pack_bf16(swiglu(bf16_lo(ga[i]), bf16_lo(ua[i])),
                             swiglu(bf16_hi(ga[i]), bf16_hi(ua[i])));
          }
          *reinterpret_cast<uint4 *>(g.out + (t_base + t) * g.ldo + static_cast<int64_t>(nt) * 64 +
                                     c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      } else {
        // KV: K3's 8-lane row code on 16 token rows at a time
        const int h = nt;   // head row of q|k|v
        const bool rotate = h < kv.Hq + kv.Hkv;
        const bool do_norm = (kv.flags & VJ_KV_NORM) != 0;
        const bool do_rope = (kv.flags & VJ_KV_ROPE) != 0;
        const int qscale =
            h < kv.Hq ? (kv.flags & (VJ_KV_QSCALE_DIV_SQRT_D | VJ_KV_QSCALE_MUL_RSQRT_D)) : 0;
        for (int row = tb + grp; row < te; row += kEpiThreads / 8) {
          const int64_t tr = t_base + row;
          const uint4 a = *reinterpret_cast<const uint4 *>(staging + stg_off(row, l8));
          const uint4 b = *reinterpret_cast<const uint4 *>(staging + stg_off(row, 8 + l8));
          RowSlice x = {{a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w}};
          if (rotate) {
            RowSlice cs{};
            if (do_rope) {
              const int pos = __ldg(kv.positions + tr);
              cs = (pos >= 0 && pos < kv.table_len)
                       ? ldg_nc_slice(reinterpret_cast<const __nv_bfloat16 *>(
                                          kv.rope_table + static_cast<int64_t>(pos) * 16), l8)
                       : rope_slice(pos, kv.rope, l8);
            }
            norm_rope_row(x, h < kv.Hq ? qw : kw, cs, grp_mask, kv.eps, do_norm, do_rope, qscale);
          }
          store_row(kv, tr, h, h < kv.Hq ? 0 : __ldg(kv.slots + tr), x, l8);
        }
      }
      named_bar_sync(1, kEpiThreads);   // staging free for the next unit
    }
  }

  tc_fence_before();
  __syncthreads();
  // peers may still read this CTA's partial buffer until they pass here
  if (g.cluster > 1) cluster_sync_all();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 256);
}

// Packed weight tiles: for weight tile nt (the rows weight_rows() names) and
// K block kb, 16 KB at ((nt * kblocks) + kb) * 16 KB holding row r's 16-byte
// chunk c at r * 128 + (c ^ (r & 7)) * 16 -- the 128-byte-swizzled K-major
// shared-memory image the MMA reads, so one bulk copy fills a stage.
__global__ void pack_tiles_kernel(const uint4 *__restrict__ w, uint4 *__restrict__ out, int k,
                                  int kblocks, int swiglu, int inter, int64_t nchunks) {
  for (int64_t o = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; o < nchunks;
       o += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tile = o >> 10;                 // 1024 chunks per tile
    const int r = static_cast<int>((o >> 3) & 127), p = static_cast<int>(o & 7);
    const int nt = static_cast<int>(tile / kblocks), kb = static_cast<int>(tile % kblocks);
    const int c = p ^ (r & 7);
    const int64_t row = swiglu ? (r < 64 ? 64 * nt + r : inter + 64 * nt + (r - 64))
                               : static_cast<int64_t>(kBN) * nt + r;
    out[o] = w[(row * k + kb * kBK + c * 8) >> 3];
  }
}

}  // namespace

namespace {

struct GemmPlan {
  int m_tiles, n_tiles, kblocks, splits, units, grid;
  int cluster;   // > 1: splits reduce through distributed shared memory
};

int set_smem_attr();

// Clusters of C CTAs of this kernel that fit on the GPU at once (cached per
// device; without a device, SMs / C).
int max_active_clusters(int C) {
  static int cache[64][kMaxCluster + 1] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return num_sms() / C;
  if (cache[dev][C] == 0) {
    int n = 0;
    if (set_smem_attr() != VJ_OK) return num_sms() / C;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(C * (num_sms() / C)), 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = static_cast<unsigned>(C);
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, decode_gemm_kernel, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms() / C;
    }
    cache[dev][C] = n;
  }
  return cache[dev][C];
}

// Work split. Automatic: the split count minimising, in units of 1/32 K
// block, (waves of units) x (K blocks per unit + ~2 for the pipeline fill and
// the epilogue) + the partial sums (~1 block per 32 tokens and split); splits
// write fp32 partials to the workspace and the last to arrive sums them. On
// request (2-8 splits at <= 64 tokens) the splits of a tile form one cluster
// and reduce through distributed shared memory instead.
GemmPlan make_plan(int64_t rows, int n_tiles, int kblocks, int splits_req) {
  GemmPlan p{};
  p.m_tiles = static_cast<int>((rows + kBM - 1) / kBM);
  p.n_tiles = n_tiles;
  p.kblocks = kblocks;
  p.cluster = 1;
  const int sms = num_sms();
  const int64_t tiles = static_cast<int64_t>(p.m_tiles) * n_tiles;
  const int64_t tokens = std::min<int64_t>(rows, kBM);
  // the cluster reduction is taken on request (an explicit split of 2-8 at
  // <= 64 tokens): measured, it does not beat the workspace reduction with the
  // deeper ring that the automatic choice keeps
  const bool clusterable = rows <= 64 && splits_req >= 2 && splits_req <= kMaxCluster;
  if (clusterable) {
    const int C = std::min(splits_req, kblocks);
    const int64_t ncl = C == 1 ? sms : std::max(1, max_active_clusters(C));
    p.splits = C;
    p.cluster = C;
    p.units = static_cast<int>(tiles * C);
    p.grid = static_cast<int>(std::min<int64_t>(tiles, ncl) * C);
    return p;
  }
  // more tiles than ticket words: no K split (such shapes fill the SMs anyway)
  const int smax = tiles > kMaxTicketTiles ? 1 : std::min(kMaxSplits, kblocks);
  int best = 1;
  if (splits_req > 0) {
    best = std::min(splits_req, smax);
  } else {
    int64_t best_cost = INT64_MAX;
    for (int s = 1; s <= smax; ++s) {
      const int64_t units = tiles * s;
      const int64_t waves = (units + sms - 1) / sms;
      const int64_t cost = 32 * waves * ((kblocks + s - 1) / s + 2) + (s - 1) * tokens;
      if (cost < best_cost) {
        best_cost = cost;
        best = s;
      }
    }
  }
  p.splits = best;
  p.units = static_cast<int>(tiles * best);
  p.grid = std::min(p.units, sms);
  return p;
}

size_t plan_workspace(const GemmPlan &p) {
  size_t b = kTicketBytes;
  if (p.splits > 1 && p.cluster == 1) {
    b += static_cast<size_t>(p.m_tiles) * p.n_tiles * p.splits * kBM * kBN * sizeof(float);
  }
  return b;
}

int set_smem_attr() {
  static bool done[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error(VJ_ERR_CUDA, "cudaGetDevice failed");
  if (dev >= 0 && dev < 64 && done[dev]) return VJ_OK;
  if (cudaFuncSetAttribute(decode_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kSmemBytes) != cudaSuccess) {
    return set_error(VJ_ERR_CUDA, "cudaFuncSetAttribute(decode_gemm_kernel) failed");
  }
  if (dev >= 0 && dev < 64) done[dev] = true;
  return VJ_OK;
}

// Shared checks and launch. n_rows_w: weight rows; n_tiles per the mode.
int launch_gemm(const char *who, const void *x, int64_t ldx, const void *w, int64_t n_rows_w,
                int32_t k, int64_t rows, int n_tiles, int32_t weight_layout, GemmArgs &g,
                const KvArgs &kv, int32_t splits, void *workspace, size_t workspace_bytes,
                int32_t *error_flag, cudaStream_t stream) {
  const std::string name(who);
  if (k <= 0 || k % kBK != 0) {
    return set_error(VJ_ERR_UNSUPPORTED, name + ": k must be a positive multiple of 64");
  }
  if (rows > 65536) return set_error(VJ_ERR_UNSUPPORTED, name + ": more than 65536 rows");
  if (splits < 0) return set_error(VJ_ERR_INVALID_ARGUMENT, name + ": splits < 0");
  if (weight_layout != VJ_WEIGHTS_ROW_MAJOR && weight_layout != VJ_WEIGHTS_TILED) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, name + ": unknown weight_layout");
  }
  if (!x || !w) return set_error(VJ_ERR_INVALID_ARGUMENT, name + ": null pointer");
  if (ldx == 0) ldx = k;
  if (ldx < k || ldx % 8 != 0 || reinterpret_cast<uintptr_t>(x) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(w) % 16 != 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     name + ": x and w must be 16-byte aligned with rows of >= k elements, "
                            "a multiple of 8");
  }
  const GemmPlan p = make_plan(rows, n_tiles, k / kBK, splits);
  // MMA N = the m tile's tokens rounded up to 16 (one x box of that many rows)
  g.n_pad = p.m_tiles == 1 ? static_cast<int>((rows + 15) / 16 * 16) : kBM;
  g.nbuf = g.n_pad <= 32 ? 8 : g.n_pad <= 64 ? 4 : 2;
  const uint32_t x_box_rows = static_cast<uint32_t>(g.n_pad);
  g.stage_bytes = static_cast<int>(kTileBytes + x_box_rows * kBK * 2);
  g.stages = std::min(kMaxStages,
                      (p.cluster > 1 ? kRingBytesCluster : kRingBytes) / g.stage_bytes);
  const size_t need = plan_workspace(p);
  if (workspace == nullptr || workspace_bytes < need ||
      reinterpret_cast<uintptr_t>(workspace) % 256 != 0) {
    return set_error(VJ_ERR_WORKSPACE, name + ": workspace of " + std::to_string(need) +
                                           " bytes (256-byte aligned) required");
  }
  CUtensorMap tmx, tmw;
  int rc = encode_tmap_3d(&tmx, x, static_cast<uint64_t>(k), static_cast<uint64_t>(rows), 1,
                          static_cast<uint64_t>(ldx) * 2, static_cast<uint64_t>(ldx) * 2 * rows,
                          kBK, x_box_rows, 1, true);
  if (rc) return rc;
  if (weight_layout == VJ_WEIGHTS_TILED) {
    memset(&tmw, 0, sizeof(tmw));   // not read: stages come from the packed tiles
    g.wtiles = static_cast<const uint8_t *>(w);
  } else {
    rc = encode_tmap_3d(&tmw, w, static_cast<uint64_t>(k), static_cast<uint64_t>(n_rows_w), 1,
                        static_cast<uint64_t>(k) * 2, static_cast<uint64_t>(k) * 2 * n_rows_w,
                        kBK, 64, 1, true);
    if (rc) return rc;
    g.wtiles = nullptr;
  }
  if ((rc = set_smem_attr()) != VJ_OK) return rc;
  g.rows = static_cast<int>(rows);
  g.kblocks = p.kblocks;
  g.m_tiles = p.m_tiles;
  g.n_tiles = p.n_tiles;
  g.splits = p.splits;
  g.cluster = p.cluster;
  g.units = p.units;
  g.tickets = static_cast<unsigned *>(workspace);
  g.partials = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + kTicketBytes);
  g.error = error_flag;
  if (p.cluster > 1) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(p.grid), 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = static_cast<unsigned>(p.cluster);
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, decode_gemm_kernel, tmx, tmw, g, kv) != cudaSuccess) {
      return set_error(VJ_ERR_CUDA, name + ": cluster launch failed: " +
                                        cudaGetErrorString(cudaGetLastError()));
    }
  } else {
    decode_gemm_kernel<<<p.grid, kGemmThreads, kSmemBytes, stream>>>(tmx, tmw, g, kv);
  }
  return check_launch(who);
}

}  // namespace
}  // namespace vj

extern "C" size_t vj_decode_gemm_workspace_size(int64_t rows, int32_t n, int32_t k, int32_t mode,
                                                int32_t splits) {
  using namespace vj;
  if (rows <= 0 || n <= 0 || k <= 0 || k % kBK != 0 || splits < 0) return 0;
  int n_tiles;
  if (mode == VJ_GEMM_SWIGLU) {
    if (n % 128 != 0) return 0;
    n_tiles = n / 128;   // (n/2) / 64
  } else {
    if (n % kBN != 0) return 0;
    n_tiles = n / kBN;
  }
  return plan_workspace(make_plan(rows, n_tiles, k / kBK, splits));
}

extern "C" vj_status vj_pack_weight_tiles(const void *w, void *out, int32_t n, int32_t k,
                                          int32_t mode, cudaStream_t stream) {
  using namespace vj;
  if (n <= 0 || k <= 0 || k % kBK != 0 || n % 128 != 0) {
    return set_error(VJ_ERR_UNSUPPORTED,
                     "vj_pack_weight_tiles: n must be a multiple of 128 and k of 64");
  }
  if (mode != VJ_GEMM_PLAIN && mode != VJ_GEMM_SWIGLU) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_pack_weight_tiles: unknown mode");
  }
  if (!w || !out || w == out || reinterpret_cast<uintptr_t>(w) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(out) % 16 != 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_pack_weight_tiles: distinct 16-byte aligned w and out required");
  }
  const int64_t nchunks = static_cast<int64_t>(n) * k / 8;
  const int grid = static_cast<int>(std::min<int64_t>((nchunks + 255) / 256, 148 * 16));
  pack_tiles_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint4 *>(w),
                                              static_cast<uint4 *>(out), k, k / kBK,
                                              mode == VJ_GEMM_SWIGLU ? 1 : 0, n / 2, nchunks);
  return check_launch("vj_pack_weight_tiles");
}

extern "C" vj_status vj_decode_gemm(const void *x, int64_t x_row_stride, const void *w,
                                    int32_t weight_layout, void *out, int64_t out_row_stride,
                                    int64_t rows, int32_t n, int32_t k, int32_t mode,
                                    int32_t splits, void *workspace, size_t workspace_bytes,
                                    int32_t *error_flag, cudaStream_t stream) {
  using namespace vj;
  if (rows < 0 || n <= 0) return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_decode_gemm: bad shape");
  if (mode != VJ_GEMM_PLAIN && mode != VJ_GEMM_SWIGLU) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_decode_gemm: unknown mode");
  }
  if (n % 128 != 0) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_decode_gemm: n must be a multiple of 128");
  }
  if (rows == 0) return VJ_OK;
  const int64_t out_cols = mode == VJ_GEMM_SWIGLU ? n / 2 : n;
  if (out_row_stride == 0) out_row_stride = out_cols;
  if (!out || out_row_stride < out_cols || out_row_stride % 8 != 0 ||
      reinterpret_cast<uintptr_t>(out) % 16 != 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_decode_gemm: out must be 16-byte aligned with a row stride >= its "
                     "columns, a multiple of 8");
  }
  GemmArgs g{};
  g.mode = mode == VJ_GEMM_SWIGLU ? kModeSwiglu : kModePlain;
  g.inter = static_cast<int>(n / 2);
  g.out = static_cast<__nv_bfloat16 *>(out);
  g.ldo = out_row_stride;
  KvArgs kv{};
  return launch_gemm("vj_decode_gemm", x, x_row_stride, w, n, k, rows,
                     mode == VJ_GEMM_SWIGLU ? n / 128 : n / kBN, weight_layout, g, kv, splits,
                     workspace, workspace_bytes, error_flag, stream);
}

extern "C" vj_status vj_qkv_gemm_kv_store(
    const void *x, int64_t x_row_stride, const void *w_qkv, int32_t weight_layout,
    const void *q_norm_w,
    const void *k_norm_w, const int32_t *positions, const int32_t *slot_mapping, void *q_out,
    void *k_cache, void *v_cache, int64_t num_tokens, int32_t hidden, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int64_t stride_block, int64_t stride_token, int64_t stride_head, const void *rope_table,
    int32_t rope_table_len, float eps, float rope_theta, int32_t flags, int32_t splits,
    void *workspace, size_t workspace_bytes, int32_t *error_flag, cudaStream_t stream) {
  using namespace vj;
  const char *who = "vj_qkv_gemm_kv_store";
  if (num_tokens < 0 || num_q_heads < 0 || num_kv_heads <= 0 || num_blocks <= 0 ||
      block_size <= 0 || rope_table_len < 0 || hidden <= 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_qkv_gemm_kv_store: negative or zero size");
  }
  if (head_dim != kHeadDim) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_qkv_gemm_kv_store: head_dim must be 128");
  }
  if ((flags & VJ_KV_QSCALE_DIV_SQRT_D) && (flags & VJ_KV_QSCALE_MUL_RSQRT_D)) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_qkv_gemm_kv_store: choose one q scaling flag");
  }
  if (num_tokens == 0) return VJ_OK;
  if (!slot_mapping || !k_cache || !v_cache || (num_q_heads > 0 && !q_out)) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_qkv_gemm_kv_store: null pointer");
  }
  if ((flags & VJ_KV_NORM) && ((num_q_heads > 0 && !q_norm_w) || !k_norm_w)) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_qkv_gemm_kv_store: VJ_KV_NORM needs norm weights");
  }
  if ((flags & VJ_KV_ROPE) && !positions) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_qkv_gemm_kv_store: VJ_KV_ROPE needs positions");
  }
  if (rope_table_len > 0 &&
      (rope_table == nullptr || reinterpret_cast<uintptr_t>(rope_table) % 16 != 0)) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_qkv_gemm_kv_store: rope_table must be 16-byte aligned");
  }
  if (reinterpret_cast<uintptr_t>(q_out) % 16 != 0 ||
      ((flags & VJ_KV_NORM) && (reinterpret_cast<uintptr_t>(q_norm_w) |
                                reinterpret_cast<uintptr_t>(k_norm_w)) % 16 != 0) ||
      (stride_block | stride_token | stride_head) % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) % 16 != 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_qkv_gemm_kv_store: q_out, norm weights and cache must be 16-byte "
                     "aligned");
  }
  const int heads = num_q_heads + 2 * num_kv_heads;
  GemmArgs g{};
  g.mode = kModeKv;
  KvArgs a{};
  a.q_w = static_cast<const __nv_bfloat16 *>(q_norm_w);
  a.k_w = static_cast<const __nv_bfloat16 *>(k_norm_w);
  a.positions = positions;
  a.slots = slot_mapping;
  a.q_out = static_cast<__nv_bfloat16 *>(q_out);
  a.k_out = nullptr;
  a.k_cache = static_cast<__nv_bfloat16 *>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16 *>(v_cache);
  a.rope_table = static_cast<const uint4 *>(rope_table);
  a.table_len = rope_table_len > 0 ? rope_table_len : 0;
  a.Hq = num_q_heads;
  a.Hkv = num_kv_heads;
  a.heads = heads;
  a.num_slots = num_blocks * block_size;
  a.block_size = block_size;
  a.bs_shift = (block_size & (block_size - 1)) == 0 ? __builtin_ctz(block_size) : -1;
  a.sb = stride_block;
  a.st = stride_token;
  a.sh = stride_head;
  a.eps = eps;
  a.flags = flags;
  build_rope_table(rope_theta, a.rope.inv_freq);
  return launch_gemm(who, x, x_row_stride, w_qkv, static_cast<int64_t>(heads) * kHeadDim, hidden,
                     num_tokens, heads, weight_layout, g, a, splits, workspace, workspace_bytes,
                     error_flag, stream);
}
