// K3: Qwen3 per-head q/k RMSNorm + interleaved-pair RoPE + KV-slot scatter in
// one pass over the projected q/k/v rows.
//
// Replaces, in the vllm-jax reference:
//   vllm/model/qwen3.py:286-296  q_norm -> apply_rope, k_norm -> apply_rope
//   vllm/model/qwen3.py:59-78    apply_rope (positions and inv_freq in bf16,
//                                pairs (x[2i], x[2i+1]), bf16 cos/sin)
//   vllm/model/qwen3.py:105-111  _update_kv_cache (.at[slot].set, mode=drop)
//   vllm/model/qwen3.py:207      decode q scaling q / bf16(sqrt(D)) (flag)
//   vllm/kernels/prefill_paged_attention.py:60  prefill q * bf16(1/sqrt(D)) (flag)
//
// Work split: 8 lanes own one 128-dim row (16 elements each, two 16-byte
// vectors), so a CTA's 256 threads work on 32 rows at a time. The main kernel
// (kv_store_tma_kernel) is persistent: a producer warp streams units of whole
// tokens (q, k, v rows and each token's (cos, sin) row of a per-position table
// built by vj_rope_table_build) through a shared-memory ring with
// cp.async.bulk, and 8 consumer warps compute and store. A register-only
// kernel (kv_store_rows_kernel) takes head counts whose units do not fit.
// The per-row arithmetic lives in kv_row.cuh, shared with the QKV GEMM
// epilogue of gemm.cu.
//
// Arithmetic per q/k element (the kernel is HBM-bound only if it issues few
// instructions per byte): squares with packed fma.rn.f32x2, norm scale
// products with mul.rn.f32x2, one cvt.rn.bf16x2 per pair, and RoPE as two
// mul.rn.bf16x2 (x1*cos, x2*sin | x1*sin, x2*cos), two byte permutes and one
// fma.rn.bf16x2 by (-1, +1). bf16 products and sums rounded once in bf16 equal
// the reference's fp32-op-then-round-to-bf16 (24 >= 2*8+2 bits: double
// rounding is innocuous for +, -, *), so every output is bit-reproducible.
#include "../../include/vjattn.h"
#include "vj_common.cuh"
#include "kv_row.cuh"

#include <algorithm>
#include <cmath>
#include <string>

namespace vj {
namespace {

constexpr int kThreads = 256;      // 32 row groups of 8 lanes

__global__ void __launch_bounds__(kThreads)
rope_table_kernel(uint32_t *table, int num_positions, RopeTable rope) {
  const int64_t n = static_cast<int64_t>(num_positions) * kPairs;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    table[i] = rope_word(static_cast<int>(i / kPairs), rope.inv_freq[i % kPairs]);
  }
}

// Register kernel (for head counts whose staged units do not fit in shared
// memory): 32 row groups per CTA, kRowsPerGrp rows each in flight.
constexpr int kRowsPerGrp = 2;
constexpr int kRowsPerCtaReg = 32 * kRowsPerGrp;

__global__ void __launch_bounds__(kThreads, 2)
kv_store_rows_kernel(const KvArgs a) {
  const int grp = threadIdx.x >> 3;
  const int l8 = threadIdx.x & 7;
  const unsigned grp_mask = 0xffu << (8 * (grp & 3));
  const bool do_norm = (a.flags & VJ_KV_NORM) != 0;
  const bool do_rope = (a.flags & VJ_KV_ROPE) != 0;
  const int qscale = a.flags & (VJ_KV_QSCALE_DIV_SQRT_D | VJ_KV_QSCALE_MUL_RSQRT_D);
  RowSlice qw, kw;
  load_weights(a, l8, qw, kw);
  for (uint32_t base = blockIdx.x * kRowsPerCtaReg; base < a.num_rows;
       base += gridDim.x * kRowsPerCtaReg) {
#pragma unroll 1
    for (int k = 0; k < kRowsPerGrp; ++k) {
      const uint32_t r = base + grp + 32 * k;
      if (r >= a.num_rows) break;
      const uint32_t tl = __umulhi(r, a.heads_magic);   // r / heads (host-checked range)
      const int h = static_cast<int>(r - tl * a.heads);
      const int64_t t = a.t_begin + tl;
      const __nv_bfloat16 *src =
          h < a.Hq ? a.q_in + t * a.qrs + h * kHeadDim
          : h < a.Hq + a.Hkv ? a.k_in + t * a.krs + (h - a.Hq) * kHeadDim
                             : a.v_in + t * a.vrs + (h - a.Hq - a.Hkv) * kHeadDim;
      RowSlice x = ldg_slice(src, l8);
      if (h < a.Hq + a.Hkv) {
        RowSlice cs{};
        if (do_rope) {
          const int pos = __ldg(a.positions + t);
          cs = (pos >= 0 && pos < a.table_len)
                   ? ldg_nc_slice(reinterpret_cast<const __nv_bfloat16 *>(
                                      a.rope_table + static_cast<int64_t>(pos) * 16), l8)
                   : rope_slice(pos, a.rope, l8);
        }
        norm_rope_row(x, h < a.Hq ? qw : kw, cs, grp_mask, a.eps, do_norm, do_rope,
                      h < a.Hq ? qscale : 0);
      }
      store_row(a, t, h, h < a.Hq ? 0 : __ldg(a.slots + t), x, l8);
    }
  }
}

// ---------------------------------------------------------------------------
// TMA-staged variant: a persistent CTA streams "units" of G whole tokens
// (G * heads rows, ~96 rows = 24 KB) through a kStages-deep shared-memory
// ring. One producer thread loads a unit's positions and slots, then issues
// untiled bulk copies (cp.async.bulk, no multicast) of its q, k and v rows and
// of its tokens' (cos, sin) table rows, counted on the stage's full barrier;
// 8 consumer warps (32 row groups of 8 lanes) normalise, rotate, scale and
// store, then release the stage. Loads of later units are in flight while a
// unit is computed, so HBM stays busy with few registers per thread.
// Every wait is bounded (2 s); a timed-out wait counts in g_kv_store_timeouts
// and the CTA drains its copies in flight and returns.
// ---------------------------------------------------------------------------
constexpr int kStages = 4;
constexpr int kConsumerWarps = 8;
constexpr int kTmaThreads = 32 * (kConsumerWarps + 1);
constexpr int kUnitRows = 96;
constexpr int kMaxUnitTokens = 32;

__device__ int g_kv_store_timeouts;

struct TmaPlan {
  int G;                 // tokens per unit
  uint32_t rows_off, tab_off, meta_off, stage_bytes;
  int64_t num_units;
};

// 9 warps of 2 CTAs share an SM: 5 warps on one sub-partition must fit its
// 16K registers, so at most 96 (allocated in steps of 8) per thread
__global__ void __maxnreg__(96)
kv_store_tma_kernel(const KvArgs a, const TmaPlan p, int64_t num_tokens) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * p.stage_bytes);
  uint64_t *empty = full + kStages;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool do_norm = (a.flags & VJ_KV_NORM) != 0;
  const bool do_rope = (a.flags & VJ_KV_ROPE) != 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    int64_t it = 0;
    bool ok = true;
    for (int64_t u = blockIdx.x; u < p.num_units; u += gridDim.x, ++it) {
      const int stage = static_cast<int>(it % kStages);
      if (it >= kStages && !mbar_wait(&empty[stage], static_cast<uint32_t>((it / kStages - 1) & 1))) {
        atomicAdd(&g_kv_store_timeouts, 1);
        ok = false;
        break;
      }
      uint8_t *base = smem + stage * p.stage_bytes;
      int2 *meta = reinterpret_cast<int2 *>(base + p.meta_off);
      const int64_t t0 = u * p.G;
      const int ng = static_cast<int>(num_tokens - t0 < p.G ? num_tokens - t0 : p.G);
      uint32_t bytes = static_cast<uint32_t>(ng) * a.heads * 256u;
#pragma unroll 4
      for (int g = 0; g < ng; ++g) {
        const int pos = do_rope ? __ldg(a.positions + t0 + g) : 0;
        meta[g] = make_int2(pos, __ldg(a.slots + t0 + g));
        if (do_rope && pos >= 0 && pos < a.table_len) bytes += 256u;
      }
      mbar_arrive_expect_tx(&full[stage], bytes);
      for (int g = 0; g < ng; ++g) {
        const int64_t t = t0 + g;
        const int pos = meta[g].x;
        uint8_t *rows = base + p.rows_off + static_cast<uint32_t>(g) * a.heads * 256u;
        if (a.Hq > 0) bulk_g2s(rows, a.q_in + t * a.qrs, a.Hq * 256u, &full[stage]);
        bulk_g2s(rows + a.Hq * 256u, a.k_in + t * a.krs, a.Hkv * 256u, &full[stage]);
        bulk_g2s(rows + (a.Hq + a.Hkv) * 256u, a.v_in + t * a.vrs, a.Hkv * 256u, &full[stage]);
        if (do_rope && pos >= 0 && pos < a.table_len) {
          bulk_g2s(base + p.tab_off + g * 256u, a.rope_table + static_cast<int64_t>(pos) * 16,
                   256u, &full[stage]);
        }
      }
    }
    // copies still in flight must land before the CTA exits (normal path: the
    // consumers already waited for all of them)
    if (!ok) {
      for (int64_t j = it > kStages ? it - kStages : 0; j < it; ++j) {
        mbar_wait(&full[j % kStages], static_cast<uint32_t>((j / kStages) & 1));
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int grp = threadIdx.x >> 3;   // 0..31
  const int l8 = threadIdx.x & 7;
  const unsigned grp_mask = 0xffu << (8 * (grp & 3));
  const int qscale = a.flags & (VJ_KV_QSCALE_DIV_SQRT_D | VJ_KV_QSCALE_MUL_RSQRT_D);
  RowSlice qw, kw;
  load_weights(a, l8, qw, kw);
  int64_t it = 0;
  for (int64_t u = blockIdx.x; u < p.num_units; u += gridDim.x, ++it) {
    const int stage = static_cast<int>(it % kStages);
    if (!mbar_wait(&full[stage], static_cast<uint32_t>((it / kStages) & 1))) {
      if (lane == 0) atomicAdd(&g_kv_store_timeouts, 1);
      return;   // without arriving: the producer's wait runs out and it drains
    }
    const uint8_t *base = smem + stage * p.stage_bytes;
    const int2 *meta = reinterpret_cast<const int2 *>(base + p.meta_off);
    const int64_t t0 = u * p.G;
    const int ng = static_cast<int>(num_tokens - t0 < p.G ? num_tokens - t0 : p.G);
    const uint32_t nrows = static_cast<uint32_t>(ng) * a.heads;
    for (uint32_t r = grp; r < nrows; r += 32) {
      const int g = static_cast<int>(__umulhi(r, a.heads_magic));   // r / heads
      const int h = static_cast<int>(r - static_cast<uint32_t>(g) * a.heads);
      RowSlice x = load_slice(base + p.rows_off + r * 256u, l8);
      if (h < a.Hq + a.Hkv) {
        RowSlice cs{};
        if (do_rope) {
          const int pos = meta[g].x;
          cs = (pos >= 0 && pos < a.table_len) ? load_slice(base + p.tab_off + g * 256u, l8)
                                                : rope_slice(pos, a.rope, l8);
        }
        norm_rope_row(x, h < a.Hq ? qw : kw, cs, grp_mask, a.eps, do_norm, do_rope,
                      h < a.Hq ? qscale : 0);
      }
      store_row(a, t0 + g, h, meta[g].y, x, l8);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
  }
}

// Unit size and shared-memory layout of the staged kernel for `heads` rows
// per token; stage_bytes == 0 when kStages stages of one token do not fit.
TmaPlan plan_tma(int heads, int64_t num_tokens) {
  TmaPlan p{};
  p.G = std::max(1, std::min(kMaxUnitTokens, kUnitRows / heads));
  const uint32_t rows = static_cast<uint32_t>(p.G) * heads * 256u;
  p.rows_off = 0;
  p.tab_off = rows;
  p.meta_off = p.tab_off + p.G * 256u;
  p.stage_bytes = (p.meta_off + p.G * 8u + 127u) & ~127u;
  if (static_cast<size_t>(kStages) * p.stage_bytes + 2 * kStages * 8 > 200 * 1024) {
    p.stage_bytes = 0;
  }
  p.num_units = (num_tokens + p.G - 1) / p.G;
  return p;
}

}  // namespace

// inv_freq = 1 / rope_theta ** (arange(0, D, 2, bf16) / D), all in bf16
// (qwen3.py:63-64). The python-float theta is weakly typed, so JAX casts it
// to bf16 before the power: theta_bf16 = bf16(rope_theta).
void build_rope_table(float rope_theta, float *inv_freq) {
  const double theta = bf16_from_f64(static_cast<double>(rope_theta));
  for (int i = 0; i < kPairs; ++i) {
    const double e = static_cast<double>(2 * i) / kHeadDim;  // exact in bf16
    const double p = bf16_from_f64(std::pow(theta, e));
    inv_freq[i] = bf16_from_f64(1.0 / p);
  }
}

}  // namespace vj

extern "C" vj_status vj_kv_store_timeouts(int32_t *count, int32_t reset) {
  using namespace vj;
  if (count == nullptr) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_kv_store_timeouts: null count");
  }
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_kv_store_timeouts, sizeof(int)) != cudaSuccess) {
    return set_error(VJ_ERR_CUDA, "vj_kv_store_timeouts: cudaMemcpyFromSymbol failed");
  }
  *count = v;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_kv_store_timeouts, &zero, sizeof(int)) != cudaSuccess) {
      return set_error(VJ_ERR_CUDA, "vj_kv_store_timeouts: cudaMemcpyToSymbol failed");
    }
  }
  return VJ_OK;
}

extern "C" size_t vj_rope_table_bytes(int32_t num_positions, int32_t head_dim) {
  if (num_positions <= 0 || head_dim != vj::kHeadDim) return 0;
  return static_cast<size_t>(num_positions) * (vj::kHeadDim / 2) * sizeof(uint32_t);
}

extern "C" vj_status vj_rope_table_build(void *table, int32_t num_positions, int32_t head_dim,
                                         float rope_theta, cudaStream_t stream) {
  using namespace vj;
  if (head_dim != kHeadDim) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_rope_table_build: head_dim must be 128, got " +
                                             std::to_string(head_dim));
  }
  if (num_positions <= 0 || table == nullptr ||
      reinterpret_cast<uintptr_t>(table) % 16 != 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_rope_table_build: need a 16-byte aligned table and num_positions > 0");
  }
  RopeTable rope;
  build_rope_table(rope_theta, rope.inv_freq);
  const int64_t n = static_cast<int64_t>(num_positions) * kPairs;
  const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 16));
  rope_table_kernel<<<grid, 256, 0, stream>>>(static_cast<uint32_t *>(table), num_positions,
                                               rope);
  return check_launch("vj_rope_table_build");
}

extern "C" vj_status vj_kv_store_qknorm_rope(
    const void *q_in, const void *k_in, const void *v_in, const void *q_norm_w,
    const void *k_norm_w, const int32_t *positions, const int32_t *slot_mapping,
    void *q_out, void *k_out, void *k_cache, void *v_cache, int64_t num_tokens,
    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
    int64_t num_blocks, int32_t block_size, int64_t stride_block,
    int64_t stride_token, int64_t stride_head, int64_t q_row_stride, int64_t k_row_stride,
    int64_t v_row_stride, const void *rope_table, int32_t rope_table_len, float eps,
    float rope_theta, int32_t flags, cudaStream_t stream) {
  using namespace vj;
  if (num_tokens < 0 || num_q_heads < 0 || num_kv_heads <= 0 || num_blocks <= 0 ||
      block_size <= 0 || rope_table_len < 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_kv_store_qknorm_rope: negative or zero size");
  }
  if (head_dim != kHeadDim) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_kv_store_qknorm_rope: head_dim must be 128, got " +
                                             std::to_string(head_dim));
  }
  const int heads = num_q_heads + 2 * num_kv_heads;
  if (heads > 4096) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_kv_store_qknorm_rope: more than 4096 head rows");
  }
  if ((flags & VJ_KV_QSCALE_DIV_SQRT_D) && (flags & VJ_KV_QSCALE_MUL_RSQRT_D)) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_kv_store_qknorm_rope: choose one q scaling flag");
  }
  if (num_tokens == 0) return VJ_OK;
  if (!k_in || !v_in || !slot_mapping || !k_cache || !v_cache ||
      (num_q_heads > 0 && (!q_in || !q_out))) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_kv_store_qknorm_rope: null pointer");
  }
  if ((flags & VJ_KV_NORM) && ((num_q_heads > 0 && !q_norm_w) || !k_norm_w)) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_kv_store_qknorm_rope: VJ_KV_NORM needs norm weights");
  }
  if ((flags & VJ_KV_ROPE) && !positions) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_kv_store_qknorm_rope: VJ_KV_ROPE needs positions");
  }
  if (rope_table_len > 0 && (rope_table == nullptr ||
                             reinterpret_cast<uintptr_t>(rope_table) % 16 != 0)) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_kv_store_qknorm_rope: rope_table must be 16-byte aligned");
  }
  if (q_row_stride == 0) q_row_stride = (int64_t)num_q_heads * kHeadDim;
  if (k_row_stride == 0) k_row_stride = (int64_t)num_kv_heads * kHeadDim;
  if (v_row_stride == 0) v_row_stride = (int64_t)num_kv_heads * kHeadDim;
  if ((q_row_stride | k_row_stride | v_row_stride) % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(q_in) | reinterpret_cast<uintptr_t>(k_in) |
       reinterpret_cast<uintptr_t>(v_in) | reinterpret_cast<uintptr_t>(q_out) |
       reinterpret_cast<uintptr_t>(k_out)) % 16 != 0 ||
      ((flags & VJ_KV_NORM) && (reinterpret_cast<uintptr_t>(q_norm_w) |
                                reinterpret_cast<uintptr_t>(k_norm_w)) % 16 != 0)) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_kv_store_qknorm_rope: q/k/v rows and weights must start on 16-byte "
                     "boundaries");
  }
  if ((stride_block | stride_token | stride_head) % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) % 16 != 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_kv_store_qknorm_rope: cache base/strides must be 16-byte aligned");
  }
  KvArgs a;
  a.q_in = static_cast<const __nv_bfloat16 *>(q_in);
  a.k_in = static_cast<const __nv_bfloat16 *>(k_in);
  a.v_in = static_cast<const __nv_bfloat16 *>(v_in);
  a.q_w = static_cast<const __nv_bfloat16 *>(q_norm_w);
  a.k_w = static_cast<const __nv_bfloat16 *>(k_norm_w);
  a.positions = positions;
  a.slots = slot_mapping;
  a.q_out = static_cast<__nv_bfloat16 *>(q_out);
  a.k_out = static_cast<__nv_bfloat16 *>(k_out);
  a.k_cache = static_cast<__nv_bfloat16 *>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16 *>(v_cache);
  a.rope_table = static_cast<const uint4 *>(rope_table);
  a.table_len = rope_table_len > 0 ? rope_table_len : 0;
  a.Hq = num_q_heads;
  a.Hkv = num_kv_heads;
  a.heads = heads;
  a.heads_magic = static_cast<uint32_t>((1ull << 32) / static_cast<uint64_t>(heads) + 1);
  a.num_slots = num_blocks * block_size;
  a.block_size = block_size;
  a.bs_shift = (block_size & (block_size - 1)) == 0 ? __builtin_ctz(block_size) : -1;
  a.sb = stride_block;
  a.st = stride_token;
  a.sh = stride_head;
  a.qrs = q_row_stride;
  a.krs = k_row_stride;
  a.vrs = v_row_stride;
  a.eps = eps;
  a.flags = flags;
  build_rope_table(rope_theta, a.rope.inv_freq);
  const TmaPlan plan = plan_tma(heads, num_tokens);
  if (plan.stage_bytes != 0) {
    // staged kernel: persistent, as many CTAs as fit on the SMs
    // the shared-memory opt-in is a per-device attribute of the kernel
    static bool smem_set[64] = {};
    const int smem = static_cast<int>(kStages * plan.stage_bytes + 2 * kStages * 8);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
      return set_error(VJ_ERR_CUDA, "vj_kv_store_qknorm_rope: cudaGetDevice failed");
    }
    if (dev < 0 || dev >= 64 || !smem_set[dev]) {
      if (cudaFuncSetAttribute(kv_store_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               200 * 1024) != cudaSuccess ||
          cudaFuncSetAttribute(kv_store_tma_kernel,
                               cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared) != cudaSuccess) {
        return set_error(VJ_ERR_CUDA, "vj_kv_store_qknorm_rope: cudaFuncSetAttribute failed");
      }
      if (dev >= 0 && dev < 64) smem_set[dev] = true;
    }
    const int per_sm = std::max(1, (227 * 1024) / (smem + 1024));
    const int64_t cap = static_cast<int64_t>(num_sms()) * per_sm;
    a.t_begin = 0;
    a.num_rows = 0;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(plan.num_units, cap));
    kv_store_tma_kernel<<<grid, kTmaThreads, smem, stream>>>(a, plan, num_tokens);
    return check_launch("vj_kv_store_qknorm_rope");
  }
  // register kernel for head counts whose stages do not fit in shared memory.
  // __umulhi(r, magic) == r / heads exactly while r * heads < 2^32 (the
  // magic's excess over 2^32 / heads is below 1): launch in token ranges
  // that keep every row index within that bound
  const int64_t max_rows = static_cast<int64_t>((1ull << 32) / static_cast<uint64_t>(heads)) - 1;
  const int64_t tokens_per_launch = std::max<int64_t>(1, max_rows / heads);
  const int64_t grid_cap = static_cast<int64_t>(num_sms()) * 8;
  for (int64_t t0 = 0; t0 < num_tokens; t0 += tokens_per_launch) {
    const int64_t nt = std::min(tokens_per_launch, num_tokens - t0);
    a.t_begin = t0;
    a.num_rows = static_cast<uint32_t>(nt * heads);
    const int64_t chunks =
        (static_cast<int64_t>(a.num_rows) + kRowsPerCtaReg - 1) / kRowsPerCtaReg;
    const unsigned grid = static_cast<unsigned>(std::min(chunks, grid_cap));
    kv_store_rows_kernel<<<grid, kThreads, 0, stream>>>(a);
    const vj_status st = check_launch("vj_kv_store_qknorm_rope");
    if (st != VJ_OK) return st;
  }
  return VJ_OK;
}
