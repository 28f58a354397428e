// K2: split-KV paged decode attention (one query token per sequence, GQA).
//
// Replaces vllm/kernels/decode_paged_attention.py:300-397 (vmap over the
// batch of paged_attention_unbatched :152-283, kernel :34-147) and its XLA
// combine :274-283, plus the bf16 q scaling at vllm/model/qwen3.py:207.
//
// Three launches on the caller's stream:
//   1. decode_plan_kernel  (1 CTA): pages per sequence, chunk size from the
//      real lengths (the reference splits by table width instead), per-
//      sequence chunk offsets, and a reset of the dynamic work counter.
//   2. decode_chunk_kernel (persistent, 2 CTAs/SM x 4 warps): each warp pulls
//      work items (chunk, kv-head) from an atomic counter and streams the
//      chunk's 16-token K/V pages through a private TMA ring (3 x 8 KB). QK^T
//      and PV run on mma.sync m16n8k16 with the GQA group as the M rows, so
//      every K/V byte is read from HBM exactly once for all g query heads.
//      Online softmax in fp32 with exp2; the quad of lanes sharing a row
//      reduces with warp shuffles. A sequence that fits one chunk writes its
//      final bf16 output directly; otherwise the chunk writes fp32 partials.
//   3. decode_combine_kernel: log-sum-exp merge of the partials (fp32).
// HBM-bound: bytes = sum(ctx)*Hkv*D*2*2 + q/out + block tables.
#include "../../include/vjattn.h"
#include "vj_common.cuh"

#include <mutex>
#include <string>

namespace vj {
namespace {
namespace dk {
#include "decode_core.cuh"
}  // namespace dk
using namespace dk;

__global__ void __launch_bounds__(kWarps * 32, kCtasPerSm)
decode_chunk_kernel(const __grid_constant__ CUtensorMap tmk,
                    const __grid_constant__ CUtensorMap tmv, DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  decode_chunk_body<kWarps>(&tmk, &tmv, a, smem, threadIdx.x >> 5, threadIdx.x & 31);
}

}  // namespace
}  // namespace vj

extern "C" size_t vj_paged_decode_workspace_size(int32_t batch, int32_t num_q_heads,
                                                 int32_t head_dim, int32_t max_chunks) {
  if (batch < 0 || num_q_heads <= 0 || head_dim != vj::kD) return 0;
  if (max_chunks <= 0) max_chunks = 4096 + batch;
  return vj::workspace_bytes(batch, num_q_heads, max_chunks);
}

namespace vj {
namespace {
vj_status decode_impl(
    const void *q, const void *k_cache, const void *v_cache, const int32_t *block_tables,
    const int32_t *context_lens, void *out, int32_t batch, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t bt_width, int32_t bt_stride, int64_t stride_block, int64_t stride_token,
    int64_t stride_head, float scale, int32_t max_chunks, void *workspace,
    size_t workspace_bytes, cudaStream_t stream, bool plan);
}  // namespace
}  // namespace vj

extern "C" vj_status vj_paged_decode(
    const void *q, const void *k_cache, const void *v_cache, const int32_t *block_tables,
    const int32_t *context_lens, void *out, int32_t batch, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t bt_width, int32_t bt_stride, int64_t stride_block, int64_t stride_token,
    int64_t stride_head, float scale, int32_t max_chunks, void *workspace,
    size_t workspace_bytes, cudaStream_t stream) {
  return vj::decode_impl(q, k_cache, v_cache, block_tables, context_lens, out, batch,
                         num_q_heads, num_kv_heads, head_dim, num_blocks, block_size, bt_width,
                         bt_stride, stride_block, stride_token, stride_head, scale, max_chunks,
                         workspace, workspace_bytes, stream, true);
}

extern "C" vj_status vj_paged_decode_planned(
    const void *q, const void *k_cache, const void *v_cache, const int32_t *block_tables,
    const int32_t *context_lens, void *out, int32_t batch, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t bt_width, int32_t bt_stride, int64_t stride_block, int64_t stride_token,
    int64_t stride_head, float scale, int32_t max_chunks, void *workspace,
    size_t workspace_bytes, cudaStream_t stream) {
  return vj::decode_impl(q, k_cache, v_cache, block_tables, context_lens, out, batch,
                         num_q_heads, num_kv_heads, head_dim, num_blocks, block_size, bt_width,
                         bt_stride, stride_block, stride_token, stride_head, scale, max_chunks,
                         workspace, workspace_bytes, stream, false);
}

namespace vj {
namespace {
vj_status decode_impl(
    const void *q, const void *k_cache, const void *v_cache, const int32_t *block_tables,
    const int32_t *context_lens, void *out, int32_t batch, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t bt_width, int32_t bt_stride, int64_t stride_block, int64_t stride_token,
    int64_t stride_head, float scale, int32_t max_chunks, void *workspace,
    size_t workspace_bytes, cudaStream_t stream, bool plan) {
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 || bt_width < 0 ||
      bt_stride < bt_width) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_paged_decode: negative or zero size");
  }
  if (num_q_heads % num_kv_heads != 0) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "vj_paged_decode: Number of Q heads must be divisible by number of KV heads. Got " +
                         std::to_string(num_q_heads) + " and " + std::to_string(num_kv_heads) + ".");
  }
  const int g = num_q_heads / num_kv_heads;
  if (head_dim != kD) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_decode: head_dim must be 128");
  }
  if (g > 8) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_decode: at most 8 query heads per KV head");
  }
  // the chunk kernel's stage words pack (kv head, chunk) as h | chunk << 8
  if (num_kv_heads > 255) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_decode: at most 255 KV heads");
  }
  if (max_chunks >= (1 << 23)) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_decode: max_chunks must be below 2^23");
  }
  if (block_size <= 0 || block_size % kPageTok != 0) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_decode: block_size must be a multiple of 16");
  }
  if (stride_block != (int64_t)block_size * stride_token) {
    return set_error(VJ_ERR_UNSUPPORTED,
                     "vj_paged_decode: tokens of a block must be evenly strided (stride_block == "
                     "block_size * stride_token)");
  }
  if (num_blocks * block_size > (int64_t)INT32_MAX) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_decode: pool larger than 2^31 slots");
  }
  if (batch == 0) return VJ_OK;
  if (!q || !k_cache || !v_cache || !block_tables || !context_lens || !out) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_paged_decode: null pointer");
  }
  if (max_chunks <= 0) max_chunks = 4096 + batch;
  if (max_chunks <= batch) {
    return set_error(VJ_ERR_INVALID_ARGUMENT, "vj_paged_decode: max_chunks must exceed batch");
  }
  const size_t need = vj::workspace_bytes(batch, num_q_heads, max_chunks);
  if (!workspace || workspace_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 16 != 0) {
    return set_error(VJ_ERR_WORKSPACE, "vj_paged_decode: workspace needs " + std::to_string(need) +
                                           " bytes, 16-byte aligned");
  }
  CUtensorMap tmk, tmv;
  const uint64_t ntok = (uint64_t)num_blocks * block_size;
  // order the two outer dims by stride (engine layout: heads inside a token row)
  const bool head_major = stride_head < stride_token;
  int rc;
  for (int i = 0; i < 2; ++i) {
    CUtensorMap *m = i ? &tmv : &tmk;
    const void *base = i ? v_cache : k_cache;
    rc = head_major ? encode_tmap_3d(m, base, kD, num_kv_heads, ntok, stride_head * 2,
                                     stride_token * 2, 64, 1, kPageTok, true)
                    : encode_tmap_3d(m, base, kD, ntok, num_kv_heads, stride_token * 2,
                                     stride_head * 2, 64, kPageTok, 1, true);
    if (rc) return rc;
  }

  DecodeArgs a;
  a.q = static_cast<const __nv_bfloat16 *>(q);
  a.out = static_cast<__nv_bfloat16 *>(out);
  a.bt = block_tables;
  a.lens = context_lens;
  a.B = batch; a.Hq = num_q_heads; a.Hkv = num_kv_heads; a.g = g;
  a.bt_stride = bt_stride;
  a.max_pages = bt_width * (block_size / kPageTok);
  a.pages_per_block = block_size / kPageTok;
  a.block_size = block_size;
  a.num_blocks = (int)num_blocks;
  a.head_major = head_major ? 1 : 0;
  a.scale_log2 = scale * kLog2e;
  a.ws = carve(workspace, batch, num_q_heads, max_chunks);

  const int grid = num_sms() * kCtasPerSm;
  if (plan) {
    decode_plan_kernel<<<1, 1024, 0, stream>>>(context_lens, batch, num_kv_heads, max_chunks,
                                               grid * kWarps, a.max_pages, a.ws);
    rc = check_launch("vj_paged_decode(plan)");
    if (rc) return rc;
  }
  const size_t smem = smem_bytes(kWarps);
  cudaFuncSetAttribute(decode_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  decode_chunk_kernel<<<grid, kWarps * 32, smem, stream>>>(tmk, tmv, a);
  rc = check_launch("vj_paged_decode(chunks)");
  if (rc) return rc;
  const int warps = batch * num_q_heads;
  decode_combine_kernel<<<(warps + 7) / 8, 256, 0, stream>>>(a);
  return check_launch("vj_paged_decode(combine)");
}
}  // namespace
}  // namespace vj

// ---------------------------------------------------------------------------
// Decode for callers that cannot allocate device memory.
//
// Some callers may not call cudaMalloc at all: a custom-call handler inside
// an XLA / JAX computation, where the runtime owns every device buffer and an
// allocation inside the handler would bypass its accounting and may
// synchronise the device, or a serving process that pins its whole memory
// budget at start-up. vj_paged_decode_noalloc takes the same inputs and
// outputs as vj_paged_decode but keeps its split-KV scratch in a fixed
// file-scope device array instead of a caller workspace.
//
// The array (kStaticScratchBytes) exists on every GPU that loads this
// library and stays allocated until the process exits. All calls on a device
// share it and it keeps the previous call's contents; the plan kernel
// rewrites every word a call reads before it is read, so nothing needs
// clearing, but two calls whose kernels overlap on the GPU (different
// streams, no ordering between them) race on the array.
// ---------------------------------------------------------------------------
namespace vj {
namespace {
constexpr size_t kStaticScratchBytes = size_t(16) << 20;  // 16 MiB per device
__device__ __align__(256) uint8_t g_decode_scratch[kStaticScratchBytes];

// The array's address belongs to a CUDA context (a module is loaded per
// context), so the cache is keyed by the current context; with the runtime's
// primary contexts that is once per device. The lookup makes no allocation.
constexpr int kMaxContexts = 128;
std::mutex g_scratch_mu;
struct ScratchEntry {
  CUcontext ctx;
  void *ptr;
};
ScratchEntry g_scratch_cache[kMaxContexts];
int g_scratch_entries = 0;
using CtxGetCurrentFn = CUresult (*)(CUcontext *);
CtxGetCurrentFn g_ctx_get_current = nullptr;

// Device address of g_decode_scratch in the current context. In host code the
// symbol only names a host-side stand-in, so the address is looked up once
// per context (with it current) and cached.
int scratch_address(void **ptr) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_ctx_get_current == nullptr) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr) {
      return set_error(VJ_ERR_CUDA, "vj_paged_decode_noalloc: cuCtxGetCurrent not found");
    }
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
  }
  CUcontext ctx = nullptr;
  void *p = nullptr;
  cudaError_t e = cudaSuccess;
  if (g_ctx_get_current(&ctx) != CUDA_SUCCESS) {
    return set_error(VJ_ERR_CUDA, "vj_paged_decode_noalloc: cuCtxGetCurrent failed");
  }
  if (ctx == nullptr) {
    // no context on this thread yet: the runtime call below creates and binds
    // the device's primary context
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || g_ctx_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
      return set_error(VJ_ERR_CUDA, "vj_paged_decode_noalloc: no CUDA context");
    }
  }
  for (int i = 0; i < g_scratch_entries; ++i) {
    if (g_scratch_cache[i].ctx == ctx) {
      *ptr = g_scratch_cache[i].ptr;
      return VJ_OK;
    }
  }
  if (g_scratch_entries == kMaxContexts) {
    return set_error(VJ_ERR_UNSUPPORTED, "vj_paged_decode_noalloc: too many CUDA contexts");
  }
  if (p == nullptr) e = cudaGetSymbolAddress(&p, g_decode_scratch);
  if (e != cudaSuccess || p == nullptr) {
    return set_error(VJ_ERR_CUDA, std::string("vj_paged_decode_noalloc: cudaGetSymbolAddress: ") +
                                      cudaGetErrorString(e));
  }
  g_scratch_cache[g_scratch_entries++] = {ctx, p};
  *ptr = p;
  return VJ_OK;
}
}  // namespace
}  // namespace vj

extern "C" size_t vj_paged_decode_noalloc_scratch_bytes(void) { return vj::kStaticScratchBytes; }

extern "C" vj_status vj_paged_decode_noalloc(
    const void *q, const void *k_cache, const void *v_cache, const int32_t *block_tables,
    const int32_t *context_lens, void *out, int32_t batch, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int64_t num_blocks, int32_t block_size,
    int32_t bt_width, int32_t bt_stride, int64_t stride_block, int64_t stride_token,
    int64_t stride_head, float scale, cudaStream_t stream) {
  using namespace vj;
  if (batch < 0 || num_q_heads <= 0 || head_dim != kD) {
    // let the shared entry point produce its usual argument message
    return vj_paged_decode(q, k_cache, v_cache, block_tables, context_lens, out, batch,
                           num_q_heads, num_kv_heads, head_dim, num_blocks, block_size, bt_width,
                           bt_stride, stride_block, stride_token, stride_head, scale, 0, nullptr,
                           0, stream);
  }
  // Largest split budget whose scratch fits the fixed array.
  const size_t per_chunk = (size_t)num_q_heads * (sizeof(float2) + sizeof(float) * kD);
  int64_t max_chunks = (int64_t)(kStaticScratchBytes / per_chunk);
  while (max_chunks > 0 &&
         vj::workspace_bytes(batch, num_q_heads, (int)max_chunks) > kStaticScratchBytes) {
    --max_chunks;
  }
  if (max_chunks <= batch) {
    return set_error(VJ_ERR_UNSUPPORTED,
                     "vj_paged_decode_noalloc: batch " + std::to_string(batch) + " with " +
                         std::to_string(num_q_heads) + " query heads needs more than the " +
                         std::to_string(kStaticScratchBytes >> 20) +
                         " MiB fixed scratch (at most " + std::to_string(max_chunks - 1) +
                         " sequences at this head count); use vj_paged_decode with a workspace");
  }
  void *scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  return vj_paged_decode(q, k_cache, v_cache, block_tables, context_lens, out, batch,
                         num_q_heads, num_kv_heads, head_dim, num_blocks, block_size, bt_width,
                         bt_stride, stride_block, stride_token, stride_head, scale,
                         (int32_t)max_chunks, scratch, kStaticScratchBytes, stream);
}
