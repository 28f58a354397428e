// Tensor-parallel all-reduce fused with the residual add and RMSNorm that
// follow o_proj and down_proj in the Qwen3 decoder layer
// (vllm/model/qwen3.py:375-389 of vllm-jax, whose model runs on one device;
// with the weights split by KV head the row-parallel GEMM outputs must be
// summed over ranks before `attn_output += x; norm`).
//
// Over NVLink peer memory: every rank's GEMM writes its partial [rows,
// hidden] into its own communication buffer (cudaIpc-shared). Each CTA of
// this kernel then announces "my partial is ready" to its counterpart CTA on
// every peer (st.release.sys of a per-CTA epoch into the peer's flag array)
// and waits, bounded by time and iterations, for theirs. A CTA works on one
// row at a time, 16 bytes per thread, with the loads of all ranks in flight
// together (plain peer loads through L2, no multicast); partials are summed
// in fp32 in rank order, so every rank gets bit-identical results, rounded to
// bf16, added to the residual in bf16, and normalised as vj_add_rmsnorm does.
//   one-shot (2 ranks): every rank reduces every row.
//   two-shot (more ranks): rank r reduces rows [r*S, (r+1)*S) into its result
//     buffer, a second CTA barrier, then every rank gathers the other slices
//     (CTA b of rank p produced exactly the rows CTA b reads from it), so each
//     rank moves 2 (N-1)/N of the data over NVLink instead of (N-1).
// The kernel never waits for a peer's kernel to FINISH; buffers alternate
// between two parities, and arriving at call i+1 proves a peer finished
// call i, so a buffer is rewritten only after every peer stopped reading it.
// The grid is fixed (4 CTAs per SM), each CTA keeps its own epoch counter, so the
// same launch can be captured in a CUDA graph and replayed.
#include "../../include/vjattn.h"
#include "vj_common.cuh"

#include <cstring>
#include <string>

namespace vj {
namespace {

constexpr int kArThreads = 256;
constexpr int kArCtasPerSm = 4;   // one row per CTA for decode batches up to 4 x SMs
constexpr int kArMaxVec = 4;        // hidden <= 8 * 256 * 4 = 8192
constexpr uint64_t kArSpinLimit = 1ull << 26;
// at most this many rows: every rank reduces every row (one barrier) even
// from 4 ranks on, where larger batches take the two-shot path
constexpr int64_t kOneShotMaxRows = 64;

struct ArArgs {
  const __nv_bfloat16 *bufs[VJ_TP_MAX_RANKS];  // partial of each rank (own included)
  __nv_bfloat16 *results[VJ_TP_MAX_RANKS];     // two-shot: reduced slice of each rank
  uint32_t *peer_flags[VJ_TP_MAX_RANKS];       // flag region in each rank's memory
  uint32_t *flags;                              // mine: [2][world][grid]
  uint32_t *epochs;                             // mine: [grid]
  int32_t *error;
  const __nv_bfloat16 *residual, *weight;
  __nv_bfloat16 *residual_out, *y;
  int rank, world, rows, hidden, two_shot;
  int gmax;   // stride of the flag arrays: the largest grid (vj_tp_grid)
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

// Cross-rank barrier between counterpart CTAs: announce `epoch` in every
// peer's flag slot (rank, b) of flag set `set`, wait (bounded) for every
// peer's announcement in mine. The release is cumulative over the CTA's
// writes that precede the __syncthreads.
VJ_DEV bool cta_barrier(const ArArgs &a, int set, uint32_t epoch, int *s_fail) {
  const int b = blockIdx.x, G = a.gmax, tid = threadIdx.x;
  const size_t base = (size_t)set * a.world * G;
  __syncthreads();
  if (tid < a.world && tid != a.rank) {
    st_release_sys(a.peer_flags[tid] + base + (size_t)a.rank * G + b, epoch);
    const uint32_t *f = a.flags + base + (size_t)tid * G + b;
    const uint64_t t0 = globaltimer_ns();
    uint64_t it = 0;
    while ((int32_t)(ld_acquire_sys(f) - epoch) < 0) {
      if (++it > kArSpinLimit || globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicExch(a.error, 1);
        *s_fail = 1;
        break;
      }
      if (it > 4096) __nanosleep(64);
    }
  }
  __syncthreads();
  return *s_fail == 0;
}

// Sum over the block of one double per thread; every thread gets the total.
VJ_DEV double block_sum(double v, double *red) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((tid & 31) == 0) red[tid >> 5] = v;
  __syncthreads();
  double t = 0.0;
#pragma unroll
  for (int w = 0; w < kArThreads / 32; ++w) t += red[w];
  __syncthreads();   // red[] is rewritten by the next row
  return t;
}

VJ_DEV double sq8(const uint32_t o[4]) {
  double ss = 0.0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const double lo = bf16_lo(o[j]), hi = bf16_hi(o[j]);
    ss += lo * lo + hi * hi;
  }
  return ss;
}

// x = residual + bf16(fp32 sum over ranks, rank order) of `row`; written to
// residual_out (and to `res`, the two-shot result buffer). Returns 1/rms.
VJ_DEV float reduce_row(const ArArgs &a, int row, __nv_bfloat16 *res, double *red) {
  const int H = a.hidden, nvec = H / 8, tid = threadIdx.x;
  const size_t off = (size_t)row * H;
  double ss = 0.0;
#pragma unroll
  for (int k = 0; k < kArMaxVec; ++k) {
    const int i = tid + k * kArThreads;
    if (i < nvec) {
      uint4 v[VJ_TP_MAX_RANKS];
#pragma unroll
      for (int r = 0; r < VJ_TP_MAX_RANKS; ++r) {
        // published by the peer's release, acquired in cta_barrier; read
        // through L2 (ld.global.cg), never from a possibly stale L1 line
        if (r < a.world) v[r] = __ldcg(reinterpret_cast<const uint4 *>(a.bufs[r] + off) + i);
      }
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
      for (int r = 0; r < VJ_TP_MAX_RANKS; ++r) {
        if (r < a.world) {
          const uint32_t w[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            acc[2 * j] += bf16_lo(w[j]);
            acc[2 * j + 1] += bf16_hi(w[j]);
          }
        }
      }
      uint32_t o[4];
      if (a.residual) {
        const uint4 xr = __ldg(reinterpret_cast<const uint4 *>(a.residual + off) + i);
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
      const uint4 xv = make_uint4(o[0], o[1], o[2], o[3]);
      reinterpret_cast<uint4 *>(a.residual_out + off)[i] = xv;
      if (res) reinterpret_cast<uint4 *>(res + off)[i] = xv;
      ss += sq8(o);
    }
  }
  const double tot = block_sum(ss, red);
  const float ms = __fdiv_rn(static_cast<float>(tot), static_cast<float>(H));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, a.eps)));
}

// y = bf16(x * (inv * w)) of `row`; x re-read from residual_out, where this
// same thread wrote it.
VJ_DEV void norm_row(const ArArgs &a, int row, float inv) {
  const int H = a.hidden, nvec = H / 8, tid = threadIdx.x;
  const size_t off = (size_t)row * H;
#pragma unroll
  for (int k = 0; k < kArMaxVec; ++k) {
    const int i = tid + k * kArThreads;
    if (i < nvec) {
      const uint4 xv = reinterpret_cast<const uint4 *>(a.residual_out + off)[i];
      const uint4 ww = __ldg(reinterpret_cast<const uint4 *>(a.weight) + i);
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w}, wws[4] = {ww.x, ww.y, ww.z, ww.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float m0 = __fmul_rn(inv, bf16_lo(wws[j])), m1 = __fmul_rn(inv, bf16_hi(wws[j]));
        o[j] = pack_bf16(__fmul_rn(bf16_lo(xw[j]), m0), __fmul_rn(bf16_hi(xw[j]), m1));
      }
      reinterpret_cast<uint4 *>(a.y + off)[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Sums over the block of one double per rank slot; every thread gets them.
VJ_DEV void block_sum_ranks(double (&v)[VJ_TP_MAX_RANKS], double *red, int world) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int r = 0; r < VJ_TP_MAX_RANKS; ++r) {
    if (r < world) {
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) v[r] += __shfl_xor_sync(0xffffffffu, v[r], o);
      if ((tid & 31) == 0) red[(tid >> 5) * VJ_TP_MAX_RANKS + r] = v[r];
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < VJ_TP_MAX_RANKS; ++r) {
    if (r < world) {
      double t = 0.0;
#pragma unroll
      for (int w = 0; w < kArThreads / 32; ++w) t += red[w * VJ_TP_MAX_RANKS + r];
      v[r] = t;
    }
  }
  __syncthreads();   // red[] is rewritten by the next rows
}

// Two-shot gather: row `j` of every peer's slice (rows [p*S, p*S + S)) is
// copied from that peer's result buffer into residual_out and normalised;
// the loads of all peers are in flight together.
VJ_DEV void gather_rows(const ArArgs &a, int j, int S, double *red) {
  const int H = a.hidden, nvec = H / 8, tid = threadIdx.x;
  double ss[VJ_TP_MAX_RANKS];
#pragma unroll
  for (int p = 0; p < VJ_TP_MAX_RANKS; ++p) ss[p] = 0.0;
#pragma unroll 1
  for (int k = 0; k < kArMaxVec; ++k) {
    const int i = tid + k * kArThreads;
    if (i < nvec) {
      uint4 xv[VJ_TP_MAX_RANKS];
#pragma unroll
      for (int p = 0; p < VJ_TP_MAX_RANKS; ++p) {
        const int row = p * S + j;
        if (p < a.world && p != a.rank && row < a.rows) {
          xv[p] = __ldcg(reinterpret_cast<const uint4 *>(a.results[p] + (size_t)row * H) + i);
        }
      }
#pragma unroll
      for (int p = 0; p < VJ_TP_MAX_RANKS; ++p) {
        const int row = p * S + j;
        if (p < a.world && p != a.rank && row < a.rows) {
          reinterpret_cast<uint4 *>(a.residual_out + (size_t)row * H)[i] = xv[p];
          const uint32_t o[4] = {xv[p].x, xv[p].y, xv[p].z, xv[p].w};
          ss[p] += sq8(o);
        }
      }
    }
  }
  block_sum_ranks(ss, red, a.world);
#pragma unroll 1
  for (int p = 0; p < a.world; ++p) {
    const int row = p * S + j;
    if (p == a.rank || row >= a.rows) continue;
    const float ms = __fdiv_rn(static_cast<float>(ss[p]), static_cast<float>(H));
    norm_row(a, row, __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, a.eps))));
  }
}

__global__ void __launch_bounds__(kArThreads, kArCtasPerSm)
allreduce_add_rmsnorm_kernel(ArArgs a) {
  const int b = blockIdx.x, G = gridDim.x, tid = threadIdx.x;
  __shared__ uint32_t s_epoch;
  __shared__ int s_fail;
  __shared__ double red[(kArThreads / 32) * VJ_TP_MAX_RANKS];
  if (tid == 0) {
    s_epoch = a.epochs[b] + 1;
    a.epochs[b] = s_epoch;
    s_fail = 0;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  // 1. every peer's partial is ready
  if (!cta_barrier(a, 0, epoch, &s_fail)) return;
  if (!a.two_shot) {
    // one-shot: every rank reduces every row
    for (int row = b; row < a.rows; row += G) norm_row(a, row, reduce_row(a, row, nullptr, red));
    return;
  }
  // two-shot: rank r reduces rows [r*S, (r+1)*S) into its result buffer ...
  const int S = (a.rows + a.world - 1) / a.world;
  const int lo = a.rank * S, hi = min(a.rows, lo + S);
  for (int row = lo + b; row < hi; row += G) {
    norm_row(a, row, reduce_row(a, row, a.results[a.rank], red));
  }
  // ... 2. every peer's slice is reduced (CTA b of rank p wrote exactly the
  // rows CTA b reads from it) ...
  if (!cta_barrier(a, 1, epoch, &s_fail)) return;
  // ... 3. and gathers the other slices (row j of every peer's slice at once)
  for (int j = b; j < S; j += G) gather_rows(a, j, S, red);
}

}  // namespace
}  // namespace vj

extern "C" int32_t vj_tp_grid(void) { return vj::kArCtasPerSm * vj::num_sms(); }

extern "C" size_t vj_tp_flags_bytes(int32_t world) {
  // flags [2][world][grid] + epochs [grid] + error word, rounded to 4 KB
  const size_t g = (size_t)vj_tp_grid();
  const size_t n = (g * (size_t)(2 * world + 1) + 1) * sizeof(uint32_t);
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
    const void *const *bufs, void *const *results, uint32_t *const *peer_flags, uint32_t *flags,
    int32_t rank, int32_t world, const void *residual, const void *weight, void *residual_out,
    void *y, int64_t rows, int32_t hidden, float eps, cudaStream_t stream) {
  using namespace vj;
  if (world < 1 || world > VJ_TP_MAX_RANKS || rank < 0 || rank >= world) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_allreduce_add_rmsnorm: bad rank/world");
  }
  if (rows < 0 || rows > INT32_MAX || hidden <= 0 || hidden % 8 ||
      hidden > 8 * kArThreads * kArMaxVec) {
    return set_error(VJ_ERR_UNSUPPORTED,
                     "vj_allreduce_add_rmsnorm: hidden must be a multiple of 8, <= 8192");
  }
  if (!bufs || !peer_flags || !flags || !weight || !y || !residual_out) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_allreduce_add_rmsnorm: null pointer");
  }
  ArArgs a{};
  for (int r = 0; r < world; ++r) {
    if (!bufs[r] || (r != rank && !peer_flags[r]) || (results && !results[r])) {
      return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_allreduce_add_rmsnorm: null peer pointer");
    }
    if ((reinterpret_cast<uintptr_t>(bufs[r]) | (results ? reinterpret_cast<uintptr_t>(results[r]) : 0)) & 15u) {
      return set_error(VJ_ERR_UNSUPPORTED, "vj_allreduce_add_rmsnorm: buffers must be 16-byte aligned");
    }
    a.bufs[r] = static_cast<const __nv_bfloat16 *>(bufs[r]);
    a.results[r] = results ? static_cast<__nv_bfloat16 *>(results[r]) : nullptr;
    a.peer_flags[r] = peer_flags[r];
  }
  const int G = vj_tp_grid();
  a.flags = flags;
  a.epochs = flags + (size_t)2 * world * G;
  a.error = reinterpret_cast<int32_t *>(flags + (size_t)(2 * world + 1) * G);
  a.residual = static_cast<const __nv_bfloat16 *>(residual);
  a.weight = static_cast<const __nv_bfloat16 *>(weight);
  a.residual_out = static_cast<__nv_bfloat16 *>(residual_out);
  a.y = static_cast<__nv_bfloat16 *>(y);
  a.rank = rank;
  a.world = world;
  a.rows = (int)rows;
  a.hidden = hidden;
  a.two_shot = results != nullptr && world > 1;
  a.eps = eps;
  // Small batches take one barrier (one-shot) even with result buffers; the
  // grid is one CTA per row a rank reduces, up to G. Every rank makes the
  // same calls with the same rows, so CTA b's epoch advances in the same
  // calls everywhere; a buffer is rewritten only after every peer has run a
  // later call (stream order: its earlier kernel had finished), whatever the
  // grid of that call.
  a.gmax = G;
  a.two_shot = a.two_shot && world > 2 && rows > kOneShotMaxRows;
  const int64_t per_rank = a.two_shot ? (rows + world - 1) / world : rows;
  const int grid = static_cast<int>(per_rank < 1 ? 1 : (per_rank < G ? per_rank : G));
  allreduce_add_rmsnorm_kernel<<<grid, kArThreads, 0, stream>>>(a);
  return check_launch("vj_allreduce_add_rmsnorm");
}
