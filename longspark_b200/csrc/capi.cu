// Library-level C-ABI entry points and the host helpers behind every kernel's
// launcher (error text, SM count, TMA descriptor encoding).
#include "common.cuh"
#include "host_common.h"

#include <mutex>
#include <string.h>

namespace ls {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int set_cuda_error(const char* what, cudaError_t e) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return LS_ERR_CUDA;
}

int host_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static void load_encode() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess) {
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
}

int encode_tma_2d_bf16(CUtensorMap* map, const void* base, long long inner, long long outer, long long pitch,
                       int box_inner, int box_outer) {
  std::call_once(g_encode_once, load_encode);
  if (g_encode == nullptr) return set_error(LS_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (no CUDA driver?)");
  if (box_inner * 2 != 128) return set_error(LS_ERR_INVALID, "TMA box inner extent must be 64 bf16 (128 B)");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((pitch * 2) & 15))
    return set_error(LS_ERR_INVALID, "TMA base must be 16-byte aligned and the row pitch a multiple of 16 bytes");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(LS_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): inner=%lld outer=%lld pitch=%lld box=%dx%d",
                     static_cast<int>(r), inner, outer, pitch, box_outer, box_inner);
  return LS_OK;
}

int encode_tma_3d_bf16(CUtensorMap* map, const void* base, long long d0, long long d1, long long d2,
                       long long stride1_bytes, long long stride2_bytes, int box0, int box1, int box2) {
  std::call_once(g_encode_once, load_encode);
  if (g_encode == nullptr) return set_error(LS_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (no CUDA driver?)");
  if (box0 * 2 != 128) return set_error(LS_ERR_INVALID, "TMA box inner extent must be 64 bf16 (128 B)");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (stride1_bytes & 15) || (stride2_bytes & 15))
    return set_error(LS_ERR_INVALID, "TMA base must be 16-byte aligned and the strides multiples of 16 bytes");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1), static_cast<cuuint64_t>(d2)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(stride1_bytes), static_cast<cuuint64_t>(stride2_bytes)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box0), static_cast<cuuint32_t>(box1), static_cast<cuuint32_t>(box2)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(LS_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d): dims %lld x %lld x %lld",
                     static_cast<int>(r), d0, d1, d2);
  return LS_OK;
}

}  // namespace ls

extern "C" int ls_version(void) { return 100; }

extern "C" const char* ls_last_error(void) { return ls::g_last_error; }

extern "C" int ls_device_sm_count(void) { return ls::host_sm_count(); }
