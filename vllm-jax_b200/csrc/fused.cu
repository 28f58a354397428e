// Fused elementwise epilogues of the Qwen3 decoder layer around the attention
// path (vllm/model/qwen3.py:375-389 and :337-341 of vllm-jax):
//   vj_add_rmsnorm  residual add + RMSNorm in one pass (input_layernorm,
//                   post_attention_layernorm and the final norm)
//   vj_silu_mul     SwiGLU activation silu(gate) * up
// Both are HBM-bound row kernels: one read and one write of each row, where
// the unfused torch sequence launched 6-8 kernels per norm at fp32.
#include "../../include/vjattn.h"
#include "vj_common.cuh"

#include <string>

namespace vj {
namespace {

constexpr int kNormThreads = 256;

// One CTA per row. r = x (+ residual) rounded to bf16 (the reference adds in
// bf16), then y = bf16(r * (rsqrt(mean(r^2) + eps) * w)) with the sum of
// squares in fp64 rounded once to fp32 (flax RMSNorm statistics in fp32).
__global__ void __launch_bounds__(kNormThreads)
add_rmsnorm_kernel(const __nv_bfloat16 *__restrict__ x, const __nv_bfloat16 *__restrict__ res,
                   const __nv_bfloat16 *__restrict__ w, __nv_bfloat16 *__restrict__ r_out,
                   __nv_bfloat16 *__restrict__ y, int H, float eps) {
  const int64_t row = blockIdx.x;
  const uint4 *xv = reinterpret_cast<const uint4 *>(x + row * H);
  const uint4 *rv = res ? reinterpret_cast<const uint4 *>(res + row * H) : nullptr;
  uint4 *rov = r_out ? reinterpret_cast<uint4 *>(r_out + row * H) : nullptr;
  const int nvec = H / 8;
  constexpr int kMaxVec = 4;  // H <= 8192 with 256 threads
  uint4 keep[kMaxVec];
  double ss = 0.0;
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int i = threadIdx.x + k * kNormThreads;
    if (i < nvec) {
      uint4 a = xv[i];
      if (rv) {
        const uint4 b = rv[i];
        uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          aw[j] = pack_bf16(bf16_lo(aw[j]) + bf16_lo(bw[j]), bf16_hi(aw[j]) + bf16_hi(bw[j]));
        }
        a = make_uint4(aw[0], aw[1], aw[2], aw[3]);
        if (rov) rov[i] = a;
      }
      keep[k] = a;
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const double lo = bf16_lo(aw[j]), hi = bf16_hi(aw[j]);
        ss += lo * lo + hi * hi;
      }
    }
  }
  __shared__ double red[kNormThreads / 32];
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < kNormThreads / 32 ? red[threadIdx.x] : 0.0;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float ms = __fdiv_rn(static_cast<float>(red[0]), static_cast<float>(H));
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
  const uint4 *wv = reinterpret_cast<const uint4 *>(w);
  uint4 *yv = reinterpret_cast<uint4 *>(y + row * H);
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int i = threadIdx.x + k * kNormThreads;
    if (i < nvec) {
      const uint4 a = keep[k], ww = __ldg(wv + i);
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, wws[4] = {ww.x, ww.y, ww.z, ww.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float m0 = __fmul_rn(inv, bf16_lo(wws[j])), m1 = __fmul_rn(inv, bf16_hi(wws[j]));
        o[j] = pack_bf16(__fmul_rn(bf16_lo(aw[j]), m0), __fmul_rn(bf16_hi(aw[j]), m1));
      }
      yv[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// out[t, i] = bf16(bf16(silu(g)) * u) with g = gu[t, i], u = gu[t, I + i].
__global__ void silu_mul_kernel(const __nv_bfloat16 *__restrict__ gu, __nv_bfloat16 *out,
                                int64_t T, int I) {
  const int64_t nvec = T * (I / 8);
  const int per_row = I / 8;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = v / per_row;
    const int c = (int)(v % per_row);
    const uint4 g = __ldg(reinterpret_cast<const uint4 *>(gu + t * 2 * I) + c);
    const uint4 u = __ldg(reinterpret_cast<const uint4 *>(gu + t * 2 * I + I) + c);
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float g0 = bf16_lo(gw[j]), g1 = bf16_hi(gw[j]);
      const float s0 = round_bf16(g0 / (1.f + expf(-g0)));
      const float s1 = round_bf16(g1 / (1.f + expf(-g1)));
      o[j] = pack_bf16(s0 * bf16_lo(uw[j]), s1 * bf16_hi(uw[j]));
    }
    reinterpret_cast<uint4 *>(out + t * I)[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace
}  // namespace vj

extern "C" vj_status vj_add_rmsnorm(const void *x, const void *residual, const void *weight,
                                    void *residual_out, void *y, int64_t rows, int32_t hidden,
                                    float eps, cudaStream_t stream) {
  using namespace vj;
  if (rows < 0 || hidden <= 0 || hidden % 8 != 0 || hidden > 8192) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_add_rmsnorm: hidden must be a multiple of 8, <= 8192");
  }
  if (rows == 0) return VJ_OK;
  if (!x || !weight || !y || (residual_out && !residual)) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_add_rmsnorm: null pointer");
  }
  if (rows > INT32_MAX) return set_error(VJ_ERR_UNSUPPORTED, "vj_add_rmsnorm: too many rows");
  add_rmsnorm_kernel<<<(unsigned)rows, kNormThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16 *>(x), static_cast<const __nv_bfloat16 *>(residual),
      static_cast<const __nv_bfloat16 *>(weight), static_cast<__nv_bfloat16 *>(residual_out),
      static_cast<__nv_bfloat16 *>(y), hidden, eps);
  return check_launch("vj_add_rmsnorm");
}

extern "C" vj_status vj_silu_mul(const void *gate_up, void *out, int64_t rows, int32_t inter,
                                 cudaStream_t stream) {
  using namespace vj;
  if (rows < 0 || inter <= 0 || inter % 8 != 0) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_silu_mul: intermediate size must be a multiple of 8");
  }
  if (rows == 0) return VJ_OK;
  if (!gate_up || !out) return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_silu_mul: null pointer");
  const int64_t nvec = rows * (inter / 8);
  int64_t grid = (nvec + 255) / 256;
  if (grid > num_sms() * 8) grid = num_sms() * 8;
  silu_mul_kernel<<<(unsigned)grid, 256, 0, stream>>>(
      static_cast<const __nv_bfloat16 *>(gate_up), static_cast<__nv_bfloat16 *>(out), rows, inter);
  return check_launch("vj_silu_mul");
}
