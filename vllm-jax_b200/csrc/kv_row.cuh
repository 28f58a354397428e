// Per-row arithmetic of K3 (q/k RMSNorm, interleaved-pair RoPE, q scaling,
// KV-slot store) shared by the K3 kernels (kv_store.cu) and the QKV GEMM
// epilogue (gemm.cu), so both produce the same bits.
//
// Reference: vllm/model/qwen3.py:59-78 (apply_rope), :105-111
// (_update_kv_cache), :286-296 (q_norm/k_norm -> apply_rope), :207 (decode q
// scaling); vllm/kernels/prefill_paged_attention.py:60 (prefill q scaling).
#pragma once

#include "../../include/vjattn.h"
#include "vj_common.cuh"

#include <string.h>

namespace vj {

// inv_freq[i] of the reference's RoPE (bf16 values), defined in kv_store.cu
void build_rope_table(float rope_theta, float *inv_freq);

namespace {

constexpr int kHeadDim = 128;
constexpr int kPairs = kHeadDim / 2;
// bf16x2 word (lo = -1.0, hi = +1.0)
constexpr uint32_t kMinusPlusOne = 0x3F80BF80u;
// bf16(1/sqrt(128)) in both halves (prefill_paged_attention.py:60)
constexpr uint32_t kRsqrtDx2 = 0x3DB53DB5u;

struct RopeTable {
  float inv_freq[kPairs];  // bf16-valued
};

struct KvArgs {
  const __nv_bfloat16 *q_in, *k_in, *v_in;
  const __nv_bfloat16 *q_w, *k_w;
  const int32_t *positions, *slots;
  __nv_bfloat16 *q_out, *k_out, *k_cache, *v_cache;
  const uint4 *rope_table;   // [table_len][16] uint4: 4 (cos,sin) bf16x2 words per lane
  int64_t t_begin;           // first token of this launch
  uint32_t num_rows;         // rows of this launch (tokens * heads)
  uint32_t heads_magic;      // floor(2^32 / heads) + 1
  int Hq, Hkv, heads;
  int table_len;
  int64_t num_slots;
  int block_size, bs_shift;  // bs_shift >= 0 when block_size is a power of two
  int64_t sb, st, sh, qrs, krs, vrs;
  float eps;
  int flags;
  RopeTable rope;
};

VJ_DEV uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
VJ_DEV uint32_t bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
VJ_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
// (lo, hi) f32 -> bf16x2 word, round to nearest even
VJ_DEV uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
// bf16x2 word -> f32x2 (lo, hi)
VJ_DEV uint64_t unpack_f32x2(uint32_t w) { return f32x2(bf16_lo(w), bf16_hi(w)); }

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

// (cos, sin) of pair i at `position` as one bf16x2 word (lo = cos, hi = sin):
// positions.astype(bf16), freqs = bf16(pos * inv_freq) (qwen3.py:62-65), trig
// in fp64 rounded once to bf16.
__device__ __noinline__ uint32_t rope_word(int position, float inv_freq) {
  const float pos = round_bf16(static_cast<float>(position));
  const float f = round_bf16(pos * inv_freq);
  double s, c;
  sincos(static_cast<double>(f), &s, &c);
  return pack_bf16(bf16_from_f64(c), bf16_from_f64(s));  // exact: bf16 values
}


// Row layout shared by both kernels: 8 lanes own one 128-dim row; lane l8
// holds dims [8*l8, 8*l8+8) and [64+8*l8, 64+8*l8+8) as 8 bf16x2 words, so
// each of the row's two 128-byte halves is one conflict-free shared-memory
// access and one coalesced global access per lane group.
struct RowSlice {
  uint32_t w[8];
};

VJ_DEV RowSlice load_slice(const void *row, int l8) {
  const uint4 a = *reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(row) + l8 * 16);
  const uint4 b =
      *reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(row) + 128 + l8 * 16);
  return {{a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w}};
}
VJ_DEV RowSlice ldg_slice(const __nv_bfloat16 *row, int l8) {
  const uint4 a = __ldcs(reinterpret_cast<const uint4 *>(row + l8 * 8));
  const uint4 b = __ldcs(reinterpret_cast<const uint4 *>(row + 64 + l8 * 8));
  return {{a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w}};
}
VJ_DEV RowSlice ldg_nc_slice(const __nv_bfloat16 *row, int l8) {
  const uint4 a = __ldg(reinterpret_cast<const uint4 *>(row + l8 * 8));
  const uint4 b = __ldg(reinterpret_cast<const uint4 *>(row + 64 + l8 * 8));
  return {{a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w}};
}
VJ_DEV void stg_slice(__nv_bfloat16 *row, int l8, const RowSlice &v, bool streaming) {
  const uint4 a = make_uint4(v.w[0], v.w[1], v.w[2], v.w[3]);
  const uint4 b = make_uint4(v.w[4], v.w[5], v.w[6], v.w[7]);
  if (streaming) {
    __stcs(reinterpret_cast<uint4 *>(row + l8 * 8), a);
    __stcs(reinterpret_cast<uint4 *>(row + 64 + l8 * 8), b);
  } else {
    *reinterpret_cast<uint4 *>(row + l8 * 8) = a;
    *reinterpret_cast<uint4 *>(row + 64 + l8 * 8) = b;
  }
}
// (cos, sin) words of the lane's 8 pairs at `position`, computed (positions
// past the end of the table)
VJ_DEV RowSlice rope_slice(int position, const RopeTable &rope, int l8) {
  RowSlice c;
#pragma unroll 1
  for (int j = 0; j < 8; ++j) {
    const int pair = (j < 4 ? 0 : 32) + l8 * 4 + (j & 3);
    c.w[j] = rope_word(position, rope.inv_freq[pair]);
  }
  return c;
}

// Norm (optional) + RoPE (optional) + q scaling (optional) of one lane's
// slice of a q or k row. The row's sum of squares is exact per bf16 square
// and summed in fp32: per lane, even and odd dims separately in word order,
// then their sum, then a butterfly over the group's 8 lanes (xor 4, 2, 1).
VJ_DEV void norm_rope_row(RowSlice &x, const RowSlice &w, const RowSlice &cs, unsigned grp_mask,
                          float eps, bool do_norm, bool do_rope, int qscale) {
  if (do_norm) {
    uint64_t xp[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) xp[j] = unpack_f32x2(x.w[j]);
    uint64_t s2 = f32x2_mul(xp[0], xp[0]);
#pragma unroll
    for (int j = 1; j < 8; ++j) s2 = f32x2_fma(xp[j], xp[j], s2);
    float se, so;
    f32x2_split(s2, se, so);
    float ss = __fadd_rn(se, so);
#pragma unroll
    for (int o = 4; o >= 1; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(grp_mask, ss, o));
    // flax RMSNorm: y = bf16(x * (rsqrt(mean(x^2) + eps) * scale)); mean = sum / 128
    // is a power-of-two scale, exact as a multiply
    const float ms = __fmul_rn(ss, 1.0f / kHeadDim);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
    const uint64_t inv2 = f32x2(inv, inv);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint64_t m = f32x2_mul(inv2, unpack_f32x2(w.w[j]));
      float y0, y1;
      f32x2_split(f32x2_mul(xp[j], m), y0, y1);
      x.w[j] = cvt_bf16x2(y0, y1);
    }
  }
  if (do_rope) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // pair (x1, x2) = word j; stack((x1*cos - x2*sin, x1*sin + x2*cos), -1)
      const uint32_t p = bf16x2_mul(x.w[j], cs.w[j]);                       // (x1 c, x2 s)
      const uint32_t q = bf16x2_mul(x.w[j], prmt(cs.w[j], cs.w[j], 0x1032)); // (x1 s, x2 c)
      const uint32_t u = prmt(p, q, 0x5410);                                // (x1 c, x1 s)
      const uint32_t v = prmt(p, q, 0x7632);                                // (x2 s, x2 c)
      x.w[j] = bf16x2_fma(v, kMinusPlusOne, u);
    }
  }
  if (qscale == VJ_KV_QSCALE_MUL_RSQRT_D) {
#pragma unroll
    for (int j = 0; j < 8; ++j) x.w[j] = bf16x2_mul(x.w[j], kRsqrtDx2);
  } else if (qscale == VJ_KV_QSCALE_DIV_SQRT_D) {
    // bf16(x / 11.3125) for every bf16 x equals bf16(fp32(x * fp32(1/11.3125)))
    // (checked exhaustively over all finite bf16 values)
    const uint64_t r2 = f32x2(1.0f / 11.3125f, 1.0f / 11.3125f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float y0, y1;
      f32x2_split(f32x2_mul(unpack_f32x2(x.w[j]), r2), y0, y1);
      x.w[j] = cvt_bf16x2(y0, y1);
    }
  }
}

// Store one finished row: q rows to q_out, k/v rows to their cache slot
// (and k rows to k_out when given).
VJ_DEV void store_row(const KvArgs &a, int64_t t, int h, int64_t slot, const RowSlice &v,
                      int l8) {
  if (h < a.Hq) {
    stg_slice(a.q_out + (t * a.Hq + h) * kHeadDim, l8, v, true);
    return;
  }
  const bool is_k = h < a.Hq + a.Hkv;
  const int hk = is_k ? h - a.Hq : h - a.Hq - a.Hkv;
  if (is_k && a.k_out != nullptr) stg_slice(a.k_out + (t * a.Hkv + hk) * kHeadDim, l8, v, false);
  if (slot < 0 && (a.flags & VJ_KV_WRAP_NEGATIVE)) slot += a.num_slots;
  if (slot < 0 || slot >= a.num_slots) return;  // mode="drop"
  const int64_t blk = a.bs_shift >= 0 ? slot >> a.bs_shift : slot / a.block_size;
  const int64_t off = a.bs_shift >= 0 ? slot & (a.block_size - 1) : slot % a.block_size;
  stg_slice((is_k ? a.k_cache : a.v_cache) + blk * a.sb + off * a.st + hk * a.sh, l8, v, false);
}

VJ_DEV void load_weights(const KvArgs &a, int l8, RowSlice &qw, RowSlice &kw) {
  for (int j = 0; j < 8; ++j) qw.w[j] = kw.w[j] = 0u;
  if (!(a.flags & VJ_KV_NORM)) return;
  if (a.Hq > 0) qw = ldg_nc_slice(a.q_w, l8);
  kw = ldg_nc_slice(a.k_w, l8);
}

}  // namespace
}  // namespace vj
