// K3: Qwen3 per-head q/k RMSNorm + interleaved-pair RoPE + KV-slot scatter in
// one pass over the projected q/k/v rows.
//
// Replaces, in the vllm-jax reference:
//   vllm/model/qwen3.py:286-296  q_norm -> apply_rope, k_norm -> apply_rope
//   vllm/model/qwen3.py:59-78    apply_rope (positions and inv_freq in bf16,
//                                pairs (x[2i], x[2i+1]), bf16 cos/sin)
//   vllm/model/qwen3.py:105-111  _update_kv_cache (.at[slot].set, mode=drop)
//
// Work split: a CTA owns one token. Every half-warp first issues the 16-byte
// loads of all its (head) rows of that token, so the loads are in flight
// together, while the first 64 threads compute the token's bf16 cos/sin pairs
// (fp64 trig, rounded once to bf16) into shared memory; then each half-warp
// normalises, rotates and stores its rows: 16 lanes x 16 bytes = one 128-dim
// head row, every global access a coalesced 16-byte vector.
// HBM-bound: each input byte is read once and each output byte written once.
#include "../../include/vjattn.h"
#include "vj_common.cuh"

#include <cmath>
#include <string>

namespace vj {
namespace {

constexpr int kThreads = 256;   // 16 half-warps
constexpr int kHeadDim = 128;
constexpr int kPairs = kHeadDim / 2;
constexpr int kRowsPerHw = 6;   // rows in flight per half-warp (96 heads per pass)

// Elementwise product of two bf16x2 words, each lane rounded to nearest even.
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

struct RopeTable {
  float inv_freq[kPairs];  // bf16-valued
};

// Round a double to the nearest bf16 (ties to even) in one step.
__host__ __device__ inline float bf16_from_f64(double x) {
#ifdef __CUDA_ARCH__
  unsigned long long b = static_cast<unsigned long long>(__double_as_longlong(x));
#else
  unsigned long long b;
  memcpy(&b, &x, sizeof(b));
#endif
  const unsigned long long lsb = (b >> 45) & 1ull;
  b += 0x00000FFFFFFFFFFFull + lsb;
  b &= ~((1ull << 45) - 1ull);
  double r;
#ifdef __CUDA_ARCH__
  r = __longlong_as_double(static_cast<long long>(b));
#else
  memcpy(&r, &b, sizeof(r));
#endif
  return static_cast<float>(r);  // exact: r has 8 significant bits
}

__global__ void __launch_bounds__(kThreads)
kv_store_qknorm_rope_kernel(const __nv_bfloat16 *__restrict__ q_in,
                            const __nv_bfloat16 *__restrict__ k_in,
                            const __nv_bfloat16 *__restrict__ v_in,
                            const __nv_bfloat16 *__restrict__ q_w,
                            const __nv_bfloat16 *__restrict__ k_w,
                            const int32_t *__restrict__ positions,
                            const int32_t *__restrict__ slots,
                            __nv_bfloat16 *q_out, __nv_bfloat16 *k_out,
                            __nv_bfloat16 *k_cache, __nv_bfloat16 *v_cache,
                            int64_t T, int Hq, int Hkv, int64_t num_slots,
                            int block_size, int64_t sb, int64_t st, int64_t sh,
                            int64_t qrs, int64_t krs, int64_t vrs,
                            float eps, int flags, RopeTable rope) {
  // per pair: bf16x2 words (cos, sin) and (sin, cos)
  __shared__ uint2 cs[kPairs];
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x;
  const bool do_norm = (flags & VJ_KV_NORM) != 0;
  const bool do_rope = (flags & VJ_KV_ROPE) != 0;
  const int heads = Hq + 2 * Hkv;
  const int hw = tid >> 4;     // half-warp index
  const int l16 = tid & 15;    // lane inside the half-warp: dims 8*l16 .. +7
  int64_t slot = slots[t];
  if (slot < 0 && (flags & VJ_KV_WRAP_NEGATIVE)) slot += num_slots;

  for (int base = 0; base < heads; base += 16 * kRowsPerHw) {
    // ---- 1. loads of this half-warp's rows, all in flight together
    uint4 raw[kRowsPerHw];
#pragma unroll
    for (int k = 0; k < kRowsPerHw; ++k) {
      const int hidx = base + hw + 16 * k;
      raw[k] = make_uint4(0u, 0u, 0u, 0u);
      if (hidx < heads) {
        const __nv_bfloat16 *src =
            hidx < Hq ? q_in + t * qrs + hidx * kHeadDim
            : hidx < Hq + Hkv ? k_in + t * krs + (hidx - Hq) * kHeadDim
                              : v_in + t * vrs + (hidx - Hq - Hkv) * kHeadDim;
        raw[k] = *reinterpret_cast<const uint4 *>(src + l16 * 8);
      }
    }
    // ---- 2. the token's cos/sin (first pass only)
    if (base == 0 && do_rope) {
      if (tid < kPairs) {
        // positions.astype(bf16); freqs = bf16(pos * inv_freq)  (qwen3.py:62-65)
        const float pos = round_bf16(static_cast<float>(positions[t]));
        const float f = round_bf16(pos * rope.inv_freq[tid]);
        double s, c;
        sincos(static_cast<double>(f), &s, &c);
        const float cb = bf16_from_f64(c), sb = bf16_from_f64(s);
        cs[tid] = make_uint2(pack_bf16(cb, sb), pack_bf16(sb, cb));  // exact: bf16 values
      }
      __syncthreads();
    }
    // ---- 3. norm, rope, stores
#pragma unroll
    for (int k = 0; k < kRowsPerHw; ++k) {
      const int hidx = base + hw + 16 * k;
      if (hidx >= heads) break;
      const int kind = hidx < Hq ? 0 : hidx < Hq + Hkv ? 1 : 2;  // q, k, v
      const int h = kind == 0 ? hidx : kind == 1 ? hidx - Hq : hidx - Hq - Hkv;
      uint32_t wd[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
      if (kind != 2) {
        const __nv_bfloat16 *w = kind == 0 ? q_w : k_w;
        if (do_norm) {
          // flax RMSNorm: y = bf16(x * (rsqrt(mean(x^2) + eps) * scale)), fp32
          double ss = 0.0;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const double lo = bf16_lo(wd[j]), hi = bf16_hi(wd[j]);
            ss += lo * lo + hi * hi;
          }
          // the two half-warps of a warp may hold different kinds of rows
          // (odd head counts under tensor parallelism): reduce within the half
          const unsigned half_mask = 0xffffu << (16 * (hw & 1));
#pragma unroll
          for (int o = 8; o >= 1; o >>= 1) ss += __shfl_xor_sync(half_mask, ss, o);
          // mean = sum / 128: a power-of-two scale, exact as a multiply
          const float ms = __fmul_rn(static_cast<float>(ss), 1.0f / kHeadDim);
          const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
          const uint4 wr = __ldg(reinterpret_cast<const uint4 *>(w + l16 * 8));
          const uint32_t ww[4] = {wr.x, wr.y, wr.z, wr.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float m0 = __fmul_rn(inv, bf16_lo(ww[j]));
            const float m1 = __fmul_rn(inv, bf16_hi(ww[j]));
            wd[j] = pack_bf16(__fmul_rn(bf16_lo(wd[j]), m0), __fmul_rn(bf16_hi(wd[j]), m1));
          }
        }
        if (do_rope) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // pair (x1, x2) = word j; stack((x1*cos - x2*sin, x1*sin + x2*cos), -1)
            // with every op rounded to bf16: the products of bf16 values are
            // exact before their rounding, so bf16x2 multiplies give the same
            // bits; the sum and difference round through fp32 as before
            const uint2 c = cs[l16 * 4 + j];
            const uint32_t ab = bf16x2_mul(wd[j], c.x);   // (x1*cos, x2*sin)
            const uint32_t de = bf16x2_mul(wd[j], c.y);   // (x1*sin, x2*cos)
            wd[j] = pack_bf16(__fsub_rn(bf16_lo(ab), bf16_hi(ab)),
                              __fadd_rn(bf16_lo(de), bf16_hi(de)));
          }
        }
      }
      const uint4 outv = make_uint4(wd[0], wd[1], wd[2], wd[3]);
      if (kind == 0) {
        *reinterpret_cast<uint4 *>(q_out + (t * Hq + h) * kHeadDim + l16 * 8) = outv;
        continue;
      }
      if (kind == 1 && k_out != nullptr) {
        *reinterpret_cast<uint4 *>(k_out + (t * Hkv + h) * kHeadDim + l16 * 8) = outv;
      }
      if (slot < 0 || slot >= num_slots) continue;  // mode="drop"
      const int64_t blk = slot / block_size, off = slot % block_size;
      __nv_bfloat16 *dst = (kind == 1 ? k_cache : v_cache) + blk * sb + off * st + h * sh;
      *reinterpret_cast<uint4 *>(dst + l16 * 8) = outv;
    }
  }
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

extern "C" vj_status vj_kv_store_qknorm_rope(
    const void *q_in, const void *k_in, const void *v_in, const void *q_norm_w,
    const void *k_norm_w, const int32_t *positions, const int32_t *slot_mapping,
    void *q_out, void *k_out, void *k_cache, void *v_cache, int64_t num_tokens,
    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
    int64_t num_blocks, int32_t block_size, int64_t stride_block,
    int64_t stride_token, int64_t stride_head, int64_t q_row_stride, int64_t k_row_stride,
    int64_t v_row_stride, float eps, float rope_theta, int32_t flags, cudaStream_t stream) {
  using namespace vj;
  if (num_tokens < 0 || num_q_heads < 0 || num_kv_heads <= 0 || num_blocks <= 0 ||
      block_size <= 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_kv_store_qknorm_rope: negative or zero size");
  }
  if (head_dim != kHeadDim) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_kv_store_qknorm_rope: head_dim must be 128, got " +
                                             std::to_string(head_dim));
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
  if (q_row_stride == 0) q_row_stride = (int64_t)num_q_heads * kHeadDim;
  if (k_row_stride == 0) k_row_stride = (int64_t)num_kv_heads * kHeadDim;
  if (v_row_stride == 0) v_row_stride = (int64_t)num_kv_heads * kHeadDim;
  if ((q_row_stride | k_row_stride | v_row_stride) % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(q_in) | reinterpret_cast<uintptr_t>(k_in) |
       reinterpret_cast<uintptr_t>(v_in)) % 16 != 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_kv_store_qknorm_rope: q/k/v rows must start on 16-byte boundaries");
  }
  if ((stride_block | stride_token | stride_head) % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) % 16 != 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_kv_store_qknorm_rope: cache base/strides must be 16-byte aligned");
  }
  RopeTable rope;
  build_rope_table(rope_theta, rope.inv_freq);
  const int64_t grid = num_tokens;
  kv_store_qknorm_rope_kernel<<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16 *>(q_in), static_cast<const __nv_bfloat16 *>(k_in),
      static_cast<const __nv_bfloat16 *>(v_in), static_cast<const __nv_bfloat16 *>(q_norm_w),
      static_cast<const __nv_bfloat16 *>(k_norm_w), positions, slot_mapping,
      static_cast<__nv_bfloat16 *>(q_out), static_cast<__nv_bfloat16 *>(k_out),
      static_cast<__nv_bfloat16 *>(k_cache), static_cast<__nv_bfloat16 *>(v_cache), num_tokens,
      num_q_heads, num_kv_heads, num_blocks * block_size, block_size, stride_block, stride_token,
      stride_head, q_row_stride, k_row_stride, v_row_stride, eps, flags, rope);
  return check_launch("vj_kv_store_qknorm_rope");
}
