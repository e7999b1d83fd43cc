// Host-side helpers shared by the C-ABI entry points: error reporting,
// argument checks, device queries and TMA descriptor creation.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/iris_b200.h"

namespace iris {

// Records the message returned by iris_last_error() (thread-local).
int set_error(int code, const char* fmt, ...);

int num_sms();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned_n(const void* p, unsigned n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

// 2-D bf16 tensor map (inner dim first) with 128-byte swizzle and the given box.
int make_tmap_2d_bf16(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int64_t row_stride_elems,
                      int box_inner, int box_outer);

// 3-D bf16 tensor map (inner, mid, outer) with 128-byte swizzle.
int make_tmap_3d_bf16(CUtensorMap* map, const void* base, int64_t d0, int64_t d1, int64_t d2, int64_t stride1_elems,
                      int64_t stride2_elems, int box0, int box1, int box2);

}  // namespace iris

#define IRIS_REQUIRE(cond, msg)                           \
  do {                                                    \
    if (!(cond)) return ::iris::set_error(IRIS_EINVAL, "%s", msg); \
  } while (0)

#define IRIS_CUDA(expr)                                                                                   \
  do {                                                                                                    \
    cudaError_t _e = (expr);                                                                              \
    if (_e != cudaSuccess) return ::iris::set_error(IRIS_ECUDA, "%s: %s", #expr, cudaGetErrorString(_e)); \
  } while (0)

#define IRIS_CHECK_STATUS(expr)   \
  do {                            \
    int _s = (expr);              \
    if (_s != IRIS_OK) return _s; \
  } while (0)
