// Host-side plumbing shared by every entry point of libvjattn: the per-thread
// last-error message, the ABI version, and tensor-map encoding through the
// driver entry point (so the library does not link libcuda directly).
#include <cudaTypedefs.h>

#include <mutex>
#include <string>

#include "../../include/vjattn.h"
#include "vj_common.cuh"

namespace vj {

static thread_local std::string g_last_error;

int set_error(int status, const std::string &msg) {
  g_last_error = msg;
  return status;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return set_error(VJ_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
  g_last_error.clear();
  return VJ_OK;
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

int encode_tmap_3d(CUtensorMap *map, const void *base, uint64_t dim0,
                   uint64_t dim1, uint64_t dim2, uint64_t stride1_bytes,
                   uint64_t stride2_bytes, uint32_t box0, uint32_t box1,
                   uint32_t box2, bool swizzle128) {
  std::call_once(g_encode_once, []() {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault,
                                &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  if (!g_encode) {
    return set_error(VJ_ERR_CUDA, "cuTensorMapEncodeTiled entry point not found");
  }
  cuuint64_t dims[3] = {dim0, dim1, dim2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {box0, box1, box2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                        const_cast<void *>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                   : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return set_error(VJ_ERR_INVALID_ARGUMENT,
                     "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) +
                         "): base/strides must be 16-byte aligned");
  }
  return VJ_OK;
}

int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  static int cached[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

}  // namespace vj

extern "C" const char *vj_get_last_error(void) { return vj::g_last_error.c_str(); }

extern "C" int vj_version(void) { return (2 << 16) | 1; }
