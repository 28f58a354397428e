// Tensor-parallel all-reduce fused with the residual add and RMSNorm that
// follow o_proj and down_proj in the Qwen3 decoder layer
// (vllm/model/qwen3.py:375-389 of vllm-jax, whose model runs on one device;
// with the weights split by KV head the row-parallel GEMM outputs must be
// summed over ranks before `attn_output += x; norm`).
//
// One-shot over NVLink peer memory: every rank's GEMM writes its partial
// [rows, hidden] into its own communication buffer (cudaIpc-shared); then
// each CTA of this kernel
//   1. announces "my partial is ready" to its counterpart CTA on every peer
//      (st.release.sys of a per-CTA epoch into the peer's flag array) and
//      waits, bounded by time and iterations, until every peer's counterpart
//      has announced the same epoch;
//   2. for its rows: loads the partial row of every rank (plain peer loads,
//      16 B per lane, no multicast), sums them in fp32 in rank order (so all
//      ranks get bit-identical results), rounds to bf16, adds the residual in
//      bf16, and applies RMSNorm exactly as vj_add_rmsnorm does;
//   3. writes the new residual and the normed row locally.
// The kernel never waits for a peer's kernel to FINISH; buffers alternate
// between two parities, and arriving at call i+1 proves a peer finished
// call i, so a buffer is rewritten only after every peer stopped reading it.
// The grid is fixed (2 x SMs), each CTA keeps its own epoch counter, so the
// same launch can be captured in a CUDA graph and replayed.
#include "../../include/vjattn.h"
#include "vj_common.cuh"

#include <cstring>
#include <string>

namespace vj {
namespace {

constexpr int kArThreads = 256;
constexpr int kArMaxVec = 4;        // hidden <= 8192
constexpr uint64_t kArSpinLimit = 1ull << 26;

struct ArArgs {
  const __nv_bfloat16 *bufs[VJ_TP_MAX_RANKS];  // partial of each rank (own included)
  uint32_t *peer_flags[VJ_TP_MAX_RANKS];       // flag array in each rank's memory
  uint32_t *flags;                              // mine: [world][grid]
  uint32_t *epochs;                             // mine: [grid]
  int32_t *error;
  const __nv_bfloat16 *residual, *weight;
  __nv_bfloat16 *residual_out, *y;
  int rank, world, rows, hidden;
  float eps;
};

VJ_DEV void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
VJ_DEV uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
VJ_DEV uint4 ld_peer16(const void *p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__global__ void __launch_bounds__(kArThreads)
allreduce_add_rmsnorm_kernel(ArArgs a) {
  const int b = blockIdx.x, G = gridDim.x, tid = threadIdx.x;
  __shared__ uint32_t s_epoch;
  __shared__ int s_fail;
  if (tid == 0) {
    s_epoch = a.epochs[b] + 1;
    a.epochs[b] = s_epoch;
    s_fail = 0;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  // 1. announce, then wait for every peer's counterpart CTA
  if (tid < a.world && tid != a.rank) {
    __threadfence_system();
    st_release_sys(a.peer_flags[tid] + (size_t)a.rank * G + b, epoch);
    const uint32_t *f = a.flags + (size_t)tid * G + b;
    const uint64_t t0 = globaltimer_ns();
    uint64_t it = 0;
    while ((int32_t)(ld_acquire_sys(f) - epoch) < 0) {
      if (++it > kArSpinLimit || globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicExch(a.error, 1);
        s_fail = 1;
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
  if (s_fail) return;

  // 2-3. rows b, b + G, ...
  const int H = a.hidden, nvec = H / 8;
  __shared__ double red[kArThreads / 32];
  for (int row = b; row < a.rows; row += G) {
    const size_t off = (size_t)row * H;
    uint4 keep[kArMaxVec];
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < kArMaxVec; ++k) {
      const int i = tid + k * kArThreads;
      if (i < nvec) {
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        for (int r = 0; r < a.world; ++r) {
          const uint4 v = ld_peer16(a.bufs[r] + off + 8 * i);
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            acc[2 * j] += bf16_lo(w[j]);
            acc[2 * j + 1] += bf16_hi(w[j]);
          }
        }
        uint32_t o[4];
        if (a.residual) {
          const uint4 xr = *reinterpret_cast<const uint4 *>(a.residual + off + 8 * i);
          const uint32_t xw[4] = {xr.x, xr.y, xr.z, xr.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // bf16(sum) + x in bf16, as the reference's `attn_output += x`
            o[j] = pack_bf16(round_bf16(acc[2 * j]) + bf16_lo(xw[j]),
                             round_bf16(acc[2 * j + 1]) + bf16_hi(xw[j]));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) o[j] = pack_bf16(acc[2 * j], acc[2 * j + 1]);
        }
        const uint4 rv = make_uint4(o[0], o[1], o[2], o[3]);
        if (a.residual_out) *reinterpret_cast<uint4 *>(a.residual_out + off + 8 * i) = rv;
        keep[k] = rv;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const double lo = bf16_lo(o[j]), hi = bf16_hi(o[j]);
          ss += lo * lo + hi * hi;
        }
      }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    if (tid < 32) {
      double v = tid < kArThreads / 32 ? red[tid] : 0.0;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (tid == 0) red[0] = v;
    }
    __syncthreads();
    const float ms = __fdiv_rn(static_cast<float>(red[0]), static_cast<float>(H));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, a.eps)));
    __syncthreads();   // red[] is rewritten by the next row
#pragma unroll
    for (int k = 0; k < kArMaxVec; ++k) {
      const int i = tid + k * kArThreads;
      if (i < nvec) {
        const uint4 xv = keep[k];
        const uint4 ww = __ldg(reinterpret_cast<const uint4 *>(a.weight) + i);
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, wws[4] = {ww.x, ww.y, ww.z, ww.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float m0 = __fmul_rn(inv, bf16_lo(wws[j])), m1 = __fmul_rn(inv, bf16_hi(wws[j]));
          o[j] = pack_bf16(__fmul_rn(bf16_lo(xw[j]), m0), __fmul_rn(bf16_hi(xw[j]), m1));
        }
        *reinterpret_cast<uint4 *>(a.y + off + 8 * i) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

}  // namespace
}  // namespace vj

extern "C" int32_t vj_tp_grid(void) { return 2 * vj::num_sms(); }

extern "C" size_t vj_tp_flags_bytes(int32_t world) {
  // flags [world][grid] + epochs [grid] + error word, rounded to 4 KB
  const size_t g = (size_t)vj_tp_grid();
  const size_t n = (g * (size_t)(world + 1) + 1) * sizeof(uint32_t);
  return (n + 4095) & ~(size_t)4095;
}

extern "C" vj_status vj_comm_alloc(size_t bytes, void **ptr) {
  using namespace vj;
  if (!ptr || bytes == 0) return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_comm_alloc: bad arguments");
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return set_error(VJ_ERR_CUDA, std::string("vj_comm_alloc: ") + cudaGetErrorString(e));
  }
  *ptr = p;
  return VJ_OK;
}

extern "C" vj_status vj_comm_free(void *ptr) {
  using namespace vj;
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return set_error(VJ_ERR_CUDA, std::string("vj_comm_free: ") + cudaGetErrorString(e));
  return VJ_OK;
}

extern "C" vj_status vj_ipc_get_handle(void *ptr, void *handle_out) {
  using namespace vj;
  if (!ptr || !handle_out) return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_ipc_get_handle: null");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) {
    return set_error(VJ_ERR_CUDA, std::string("vj_ipc_get_handle: ") + cudaGetErrorString(e));
  }
  static_assert(sizeof(h) == VJ_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  return VJ_OK;
}

extern "C" vj_status vj_ipc_open_handle(const void *handle, void **ptr) {
  using namespace vj;
  if (!ptr || !handle) return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_ipc_open_handle: null");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    return set_error(VJ_ERR_CUDA, std::string("vj_ipc_open_handle: ") + cudaGetErrorString(e));
  }
  return VJ_OK;
}

extern "C" vj_status vj_ipc_close_handle(void *ptr) {
  using namespace vj;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    return set_error(VJ_ERR_CUDA, std::string("vj_ipc_close_handle: ") + cudaGetErrorString(e));
  }
  return VJ_OK;
}

extern "C" vj_status vj_allreduce_add_rmsnorm(
    const void *const *bufs, uint32_t *const *peer_flags, uint32_t *flags, int32_t rank,
    int32_t world, const void *residual, const void *weight, void *residual_out, void *y,
    int64_t rows, int32_t hidden, float eps, cudaStream_t stream) {
  using namespace vj;
  if (world < 1 || world > VJ_TP_MAX_RANKS || rank < 0 || rank >= world) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_allreduce_add_rmsnorm: bad rank/world");
  }
  if (rows < 0 || rows > INT32_MAX || hidden <= 0 || hidden % 8 || hidden > 8 * kArThreads * kArMaxVec) {
    return set_error(VJ_ERR_UNSUPPORTED,
                     "vj_allreduce_add_rmsnorm: hidden must be a multiple of 8, <= 8192");
  }
  if (!bufs || !peer_flags || !flags || !weight || !y) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_allreduce_add_rmsnorm: null pointer");
  }
  ArArgs a{};
  for (int r = 0; r < world; ++r) {
    if (!bufs[r] || (r != rank && !peer_flags[r])) {
      return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_allreduce_add_rmsnorm: null peer pointer");
    }
    if (reinterpret_cast<uintptr_t>(bufs[r]) & 15u) {
      return set_error(VJ_ERR_UNSUPPORTED, "vj_allreduce_add_rmsnorm: buffers must be 16-byte aligned");
    }
    a.bufs[r] = static_cast<const __nv_bfloat16 *>(bufs[r]);
    a.peer_flags[r] = peer_flags[r];
  }
  const int G = vj_tp_grid();
  a.flags = flags;
  a.epochs = flags + (size_t)world * G;
  a.error = reinterpret_cast<int32_t *>(flags + (size_t)(world + 1) * G);
  a.residual = static_cast<const __nv_bfloat16 *>(residual);
  a.weight = static_cast<const __nv_bfloat16 *>(weight);
  a.residual_out = static_cast<__nv_bfloat16 *>(residual_out);
  a.y = static_cast<__nv_bfloat16 *>(y);
  a.rank = rank;
  a.world = world;
  a.rows = (int)rows;
  a.hidden = hidden;
  a.eps = eps;
  // every call launches the same grid, even with no rows: the per-CTA epochs
  // and the peers' waits must advance together on all ranks
  allreduce_add_rmsnorm_kernel<<<G, kArThreads, 0, stream>>>(a);
  return check_launch("vj_allreduce_add_rmsnorm");
}
