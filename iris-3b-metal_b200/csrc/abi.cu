// Library plumbing behind the C ABI: last-error messages, the device error
// word, SM count and TMA descriptor creation (driver entry point looked up at
// run time, so the library links only against the CUDA runtime).
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "iris_abi_internal.h"

namespace iris {

namespace {
thread_local char g_message[512] = "";

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}
}  // namespace

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_message, sizeof(g_message), fmt, ap);
  va_end(ap);
  return code;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 64 && cache[dev] > 0) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  if (dev < 64) cache[dev] = n;
  return n;
}

int make_tmap_2d_bf16(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int64_t row_stride_elems,
                      int box_inner, int box_outer) {
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(IRIS_ECUDA, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_elems * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(IRIS_ECUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return IRIS_OK;
}

int make_tmap_3d_bf16(CUtensorMap* map, const void* base, int64_t d0, int64_t d1, int64_t d2, int64_t stride1_elems,
                      int64_t stride2_elems, int box0, int box1, int box2) {
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(IRIS_ECUDA, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1), static_cast<cuuint64_t>(d2)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(stride1_elems * 2), static_cast<cuuint64_t>(stride2_elems * 2)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box0), static_cast<cuuint32_t>(box1), static_cast<cuuint32_t>(box2)};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(IRIS_ECUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return IRIS_OK;
}

}  // namespace iris

extern "C" const char* iris_last_error(void) { return iris::g_message; }

extern "C" int iris_abi_version(void) { return 1; }

extern "C" int iris_device_error(int clear, unsigned int* value, void* stream) {
  IRIS_REQUIRE(value != nullptr, "iris_device_error: null output");
  IRIS_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  unsigned int v = 0;
  IRIS_CUDA(cudaMemcpyFromSymbol(&v, iris::g_device_error, sizeof(v)));
  if (clear) {
    unsigned int zero = 0;
    IRIS_CUDA(cudaMemcpyToSymbol(iris::g_device_error, &zero, sizeof(zero)));
  }
  *value = v;
  return IRIS_OK;
}
