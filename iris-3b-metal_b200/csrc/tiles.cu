// Tiled one-step restoration around the denoiser (the restoration / 4x
// upscaling task: tiled() and gaussian_window() of
// src/iris3b/downstream/restoration.py:75-101, restore_tile of
// src/iris_metal/tasks.py:143-150):
//
//   tile_crop         one tile x tile crop of a [C, H, W] image into a batch slot
//   tile_accumulate   out[crop] += (x[crop] - sigma v) * window, weight[crop] += window
//                     (the restored tile and its Gaussian-window fusion in one pass)
//   tile_normalize    out /= weight
//
// All fp32, one thread per pixel (channels looped inside), coalesced along W.
#include "common.cuh"
#include "iris_abi_internal.h"

namespace iris {
namespace tiles {

constexpr int THREADS = 256;

inline unsigned grid_for(int64_t n) {
  int64_t blocks = (n + THREADS - 1) / THREADS;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
  if (blocks < 1) blocks = 1;
  return static_cast<unsigned>(blocks < cap ? blocks : cap);
}

__global__ void crop_kernel(const float* __restrict__ x, int channels, int64_t height, int64_t width, int64_t top,
                            int64_t left, int64_t tile, float* __restrict__ out) {
  const int64_t total = channels * tile * tile;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t j = e % tile, i = (e / tile) % tile, c = e / (tile * tile);
    out[e] = x[(c * height + top + i) * width + left + j];
  }
}

__global__ void accumulate_kernel(const float* __restrict__ x, int channels, int64_t height, int64_t width,
                                  const float* __restrict__ v, int64_t tile, const float* __restrict__ window,
                                  int64_t top, int64_t left, float sigma, float* __restrict__ out,
                                  float* __restrict__ weight) {
  const int64_t pixels = tile * tile;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < pixels;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = e / tile, j = e % tile;
    const float w = window[e];
    const int64_t p = (top + i) * width + left + j;
    if (v != nullptr) {
      for (int c = 0; c < channels; ++c) {
        const int64_t at = static_cast<int64_t>(c) * height * width + p;
        out[at] += (x[at] - sigma * v[static_cast<int64_t>(c) * pixels + e]) * w;
      }
    }
    if (weight != nullptr) weight[p] += w;
  }
}

__global__ void normalize_kernel(float* __restrict__ out, const float* __restrict__ weight, int channels,
                                 int64_t plane) {
  const int64_t total = channels * plane;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[e] /= weight[e % plane];
}

}  // namespace tiles
}  // namespace iris

using namespace iris;

extern "C" int iris_tile_crop(const float* x, int64_t channels, int64_t height, int64_t width, int64_t top,
                              int64_t left, int64_t tile, float* out, void* stream) {
  using namespace iris::tiles;
  IRIS_REQUIRE(x && out, "tile_crop: null pointer");
  IRIS_REQUIRE(channels > 0 && tile > 0 && top >= 0 && left >= 0 && top + tile <= height && left + tile <= width,
               "tile_crop: the tile must lie inside the image");
  crop_kernel<<<grid_for(channels * tile * tile), THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      x, static_cast<int>(channels), height, width, top, left, tile, out);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_tile_accumulate(const float* x, int64_t channels, int64_t height, int64_t width, const float* v,
                                    int64_t tile, const float* window, int64_t top, int64_t left, float sigma,
                                    float* out, float* weight, void* stream) {
  using namespace iris::tiles;
  IRIS_REQUIRE(window != nullptr, "tile_accumulate: null window");
  IRIS_REQUIRE(v == nullptr || (x != nullptr && out != nullptr), "tile_accumulate: a tile needs x and out");
  IRIS_REQUIRE(v != nullptr || weight != nullptr, "tile_accumulate: nothing to accumulate");
  IRIS_REQUIRE(channels > 0 && tile > 0 && top >= 0 && left >= 0 && top + tile <= height && left + tile <= width,
               "tile_accumulate: the tile must lie inside the image");
  accumulate_kernel<<<grid_for(tile * tile), THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      x, static_cast<int>(channels), height, width, v, tile, window, top, left, sigma, out, weight);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_tile_normalize(float* out, const float* weight, int64_t channels, int64_t height, int64_t width,
                                   void* stream) {
  using namespace iris::tiles;
  IRIS_REQUIRE(out && weight, "tile_normalize: null pointer");
  IRIS_REQUIRE(channels > 0 && height > 0 && width > 0, "tile_normalize: empty image");
  normalize_kernel<<<grid_for(channels * height * width), THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      out, weight, static_cast<int>(channels), height * width);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}
