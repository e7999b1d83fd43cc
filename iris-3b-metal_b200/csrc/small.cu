// Layout, conditioning and sampler kernels around the trunk:
//   patchify / unpatchify    integer index maps (bit-exact), dit.py:326, 367-374
//   block_copy               strided block gather/scatter: the sequence-parallel
//                            (Ulysses) packing around the all-to-all exchanges
//   timestep_embedding       src/iris3b/nn/embeddings.py:41-45
//   gemv                     small-M linear (conditioning MLP, shared adaLN cores)
//   add_bias_rows            SharedCoreBias, src/iris3b/nn/modulation.py:284-285
//   cfg_euler                CFG combine + flow-Euler step, solver.py:72-74, sampling.py:129-135
//   dpm_update               CFG combine + x0 prediction + DPM-Solver++ (1st/2nd order) step,
//                            src/iris3b/flow/solver.py:58-109
//   all_finite               require_finite, src/iris_metal/model.py:102-110
//   poison_on_error          NaN-fill of a result computed after a timed-out bounded wait
#include "common.cuh"
#include "iris_abi_internal.h"

namespace iris {
namespace small {

constexpr int THREADS = 256;

inline unsigned grid_for(int64_t n, int per_thread = 1) {
  int64_t blocks = (n + static_cast<int64_t>(THREADS) * per_thread - 1) / (static_cast<int64_t>(THREADS) * per_thread);
  const int64_t cap = static_cast<int64_t>(num_sms()) * 32;
  if (blocks < 1) blocks = 1;
  return static_cast<unsigned>(blocks < cap ? blocks : cap);
}

// out[(b, l - token_start), (c, ky, kx)] = x[b, c, gy p + ky, gx p + kx] for the
// patch tokens l = gy * gw + gx in [token_start, token_start + tokens). A block
// walks whole token rows (grid-stride): the row's image position is worked out
// once, and consecutive threads take consecutive features, so a warp reads
// runs of a patch row and writes one contiguous run of the token row.
__global__ void patchify_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ out, int64_t rows,
                                int channels, int64_t height, int64_t width, int patch, int64_t token_start,
                                int64_t tokens) {
  const int64_t gw = width / patch;
  const int pp = patch * patch;
  const int feat = channels * pp;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t b = row / tokens, l = token_start + (row - b * tokens);
    const int64_t gy = l / gw, gx = l - gy * gw;
    const float* src = x + b * channels * height * width + gy * patch * width + gx * patch;
    __nv_bfloat16* dst = out + row * feat;
    for (int f = threadIdx.x; f < feat; f += blockDim.x) {
      const int c = f / pp, k = f - c * pp;
      const int ky = k / patch;
      dst[f] = __float2bfloat16_rn(src[(static_cast<int64_t>(c) * height + ky) * width + (k - ky * patch)]);
    }
  }
}

// v[b, c, y, x] = out[(b, gy, gx), ky p + kx, c]
__global__ void unpatchify_kernel(const float* __restrict__ src, float* __restrict__ v, int64_t total, int channels,
                                  int64_t height, int64_t width, int patch) {
  const int64_t gw = width / patch, L = (height / patch) * gw;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t xx = i % width;
    const int64_t y = (i / width) % height;
    const int64_t c = (i / (width * height)) % channels;
    const int64_t b = i / (width * height * channels);
    const int64_t l = (y / patch) * gw + xx / patch;
    const int64_t k = (y % patch) * patch + xx % patch;
    v[i] = src[((b * L + l) * patch * patch + k) * channels + c];
  }
}

__global__ void timestep_kernel(const float* __restrict__ t, float* __restrict__ out, int64_t batch, int half,
                                float log_period) {
  const int64_t total = batch * half;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = i / half;
    const int k = static_cast<int>(i % half);
    // the fp32 argument -ln(max_period) * k / n as the reference forms it; exp,
    // cos and sin evaluated in double and rounded once, so phases of up to
    // 1000 rad match the reference's fp32 values to the last ulp
    const float arg = (-log_period * static_cast<float>(k)) / static_cast<float>(half);
    const float freq = static_cast<float>(exp(static_cast<double>(arg)));
    const float phase = t[b] * freq;
    out[b * 2 * half + k] = static_cast<float>(cos(static_cast<double>(phase)));
    out[b * 2 * half + half + k] = static_cast<float>(sin(static_cast<double>(phase)));
  }
}

IRIS_DEVICE float silu(float v) { return v / (1.f + __expf(-v)); }

// Small-M linear, HBM-bound on the weights. Each warp owns COLS output columns
// at a time and walks K in 256-wide chunks (elements [8 l, 8 l + 8) of each
// chunk per lane). A warp's column groups (grid-stride over the columns, the
// grid sized to the blocks resident at once) and their chunks form one stream
// of weight loads with GEMV_DEPTH chunks in flight, so the stream runs on from
// one group into the next. act_in(x) of MT rows (all of K) is staged once per
// block in shared memory; more rows take further passes over the weights.
constexpr int GEMV_CHUNK = 256;
constexpr int GEMV_DEPTH = 4;

template <typename TW>
struct GemvVec;
template <>
struct GemvVec<__nv_bfloat16> {
  uint4 u;
  IRIS_DEVICE void load(const __nv_bfloat16* p, bool ok) {
    u = ok ? __ldg(reinterpret_cast<const uint4*>(p)) : make_uint4(0u, 0u, 0u, 0u);
  }
  IRIS_DEVICE void get(float (&v)[8]) const {
    const uint32_t ws[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float2 f = unpack_bf16x2(ws[h]);
      v[2 * h] = f.x;
      v[2 * h + 1] = f.y;
    }
  }
};
template <>
struct GemvVec<float> {
  float4 a, b;
  IRIS_DEVICE void load(const float* p, bool ok) {
    a = ok ? __ldg(reinterpret_cast<const float4*>(p)) : make_float4(0.f, 0.f, 0.f, 0.f);
    b = ok ? __ldg(reinterpret_cast<const float4*>(p) + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  IRIS_DEVICE void get(float (&v)[8]) const {
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
};

template <typename TW, int COLS, int MT>
__global__ void __launch_bounds__(THREADS, 2)
    gemv_kernel(const float* __restrict__ x, int M, int K, const TW* __restrict__ w, const float* __restrict__ bias,
                float* __restrict__ out, int N, int act_in, int act_out) {
  extern __shared__ __align__(16) float xs[];  // [MT][K]
  constexpr int WARPS = THREADS / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int chunks = (K + GEMV_CHUNK - 1) / GEMV_CHUNK;
  const int groups = (N + COLS - 1) / COLS;
  const int stride = gridDim.x * WARPS;  // groups between a warp's consecutive groups
  const int g0 = blockIdx.x * WARPS + warp;
  const int items = g0 < groups ? ((groups - 1 - g0) / stride + 1) * chunks : 0;  // (group, chunk) pairs
  for (int m0 = 0; m0 < M; m0 += MT) {
    const int mt = min(MT, M - m0);
    __syncthreads();  // the previous pass's readers are done with xs
    for (int e = threadIdx.x * 4; e < mt * K; e += THREADS * 4) {  // K % 8 == 0: whole float4s
      float4 v = __ldg(reinterpret_cast<const float4*>(x + static_cast<int64_t>(m0) * K + e));
      if (act_in) v = make_float4(silu(v.x), silu(v.y), silu(v.z), silu(v.w));
      *reinterpret_cast<float4*>(xs + e) = v;
    }
    __syncthreads();
    float acc[COLS][MT];
#pragma unroll
    for (int c = 0; c < COLS; ++c)
#pragma unroll
      for (int j = 0; j < MT; ++j) acc[c][j] = 0.f;
    GemvVec<TW> wq[GEMV_DEPTH][COLS];
    // the load stream's position: item, its group's first column and its chunk
    int l_item = 0, l_n0 = g0 * COLS, l_chunk = 0;
    auto load = [&](GemvVec<TW> (&dst)[COLS]) {
      const int k = l_chunk * GEMV_CHUNK + lane * 8;
#pragma unroll
      for (int c = 0; c < COLS; ++c)
        dst[c].load(w + static_cast<int64_t>(l_n0 + c) * K + k, l_item < items && l_n0 + c < N && k < K);
      ++l_item;
      if (++l_chunk == chunks) {
        l_chunk = 0;
        l_n0 += stride * COLS;
      }
    };
#pragma unroll
    for (int d = 0; d < GEMV_DEPTH; ++d) load(wq[d]);
    // the compute stream's position
    int c_n0 = g0 * COLS, c_chunk = 0;
    for (int it = 0; it < items; it += GEMV_DEPTH) {
#pragma unroll
      for (int d = 0; d < GEMV_DEPTH; ++d) {
        if (it + d < items) {  // warp-uniform
          const int k = c_chunk * GEMV_CHUNK + lane * 8;
          if (k < K) {
            float wv[COLS][8];
#pragma unroll
            for (int c = 0; c < COLS; ++c) wq[d][c].get(wv[c]);
#pragma unroll
            for (int j = 0; j < MT; ++j) {
              if (j < mt) {
                const float4 a = *reinterpret_cast<const float4*>(xs + j * K + k);
                const float4 b = *reinterpret_cast<const float4*>(xs + j * K + k + 4);
                const float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
                for (int c = 0; c < COLS; ++c)
#pragma unroll
                  for (int e = 0; e < 8; ++e) acc[c][j] = fmaf(xv[e], wv[c][e], acc[c][j]);
              }
            }
          }
          if (++c_chunk == chunks) {  // the group's columns are complete
#pragma unroll
            for (int c = 0; c < COLS; ++c) {
#pragma unroll
              for (int j = 0; j < MT; ++j) {
                if (j < mt) {
                  const float sum = warp_sum(acc[c][j]);
                  if (lane == 0 && c_n0 + c < N) {
                    const float r = sum + (bias ? bias[c_n0 + c] : 0.f);
                    out[static_cast<int64_t>(m0 + j) * N + c_n0 + c] = act_out ? silu(r) : r;
                  }
                }
                acc[c][j] = 0.f;
              }
            }
            c_chunk = 0;
            c_n0 += stride * COLS;
          }
        }
        load(wq[d]);
      }
    }
  }
}

__global__ void add_bias_rows_kernel(const float* __restrict__ core, const float* __restrict__ bias,
                                     float* __restrict__ out, int64_t batch, int64_t n_blocks, int64_t width) {
  const int64_t total = n_blocks * batch * width;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = i % width;
    const int64_t b = (i / width) % batch;
    const int64_t j = i / (width * batch);
    out[i] = core[b * width + e] + bias[j * width + e];
  }
}

__global__ void cfg_euler_kernel(const float* __restrict__ v, const float* __restrict__ x, float* __restrict__ x_out,
                                 int64_t images, int64_t per_image, float cfg_scale, float sigma, float sigma_next,
                                 int guided) {
  const int64_t total = images * per_image;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float vel;
    if (guided) {
      const float u = v[i], c = v[total + i];
      vel = u + cfg_scale * (c - u);
    } else {
      vel = v[i];
    }
    const float xi = x[i];
    const float clean = xi - sigma * vel;
    if (sigma_next < 0.f) {
      x_out[i] = clean;
    } else {
      const float implied = (xi - (1.f - sigma) * clean) / sigma;
      x_out[i] = (1.f - sigma_next) * clean + sigma_next * implied;
    }
  }
}

// One multistep DPM-Solver++ step on the rectified-flow schedule
// (src/iris3b/flow/solver.py:58-109): out = v_u + g (v_c - v_u) (guided) or v;
// x0 = out (x-prediction) or x - s out (v-prediction);
// x_out = a x + b x0 + c (x0 - x0_prev) (c = 0: first order, x0_prev unused).
// x0 is written to x0_out for the next step's history.
__global__ void dpm_update_kernel(const float* __restrict__ v, const float* __restrict__ x,
                                  const float* __restrict__ x0_prev, float* __restrict__ x0_out,
                                  float* __restrict__ x_out, int64_t total, float cfg_scale, int guided,
                                  float sigma, int predict_x, float a, float b, float c) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float out;
    if (guided) {
      const float u = v[i], w = v[total + i];
      out = u + cfg_scale * (w - u);
    } else {
      out = v[i];
    }
    const float xi = x[i];
    const float x0 = predict_x ? out : xi - sigma * out;
    float xn = a * xi + b * x0;
    if (x0_prev != nullptr) xn += c * (x0 - x0_prev[i]);
    x0_out[i] = x0;
    x_out[i] = xn;
  }
}

__global__ void all_finite_kernel(const float* __restrict__ x, int64_t n, int* flag) {
  int bad = 0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    bad |= !isfinite(x[i]);
  bad = __syncthreads_or(bad);
  if (bad && threadIdx.x == 0) atomicExch(flag, 0);
}

__global__ void set_int_kernel(int* p, int v) { *p = v; }

// x[i] = NaN for every i when the device error word has a bit of `mask` set
// (a bounded wait gave up earlier on this device); otherwise every thread
// reads the word once and leaves.
__global__ void poison_on_error_kernel(float* __restrict__ x, int64_t n, unsigned int mask) {
  if ((*reinterpret_cast<volatile unsigned int*>(&g_device_error) & mask) == 0u) return;
  const float nan = __int_as_float(0x7fc00000);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    x[i] = nan;
}

// Block (i0, i1, i2) of `vecs` 16-byte vectors: src + i0 s0 + i1 s1 + i2 s2 ->
// dst + i0 d0 + i1 d1 + i2 d2 (byte strides). One CTA item = 1024 vectors of a
// block, 4 per thread with all loads issued before the stores.
constexpr int COPY_VECS_PER_THREAD = 4;
constexpr int COPY_CHUNK = THREADS * COPY_VECS_PER_THREAD;

__global__ void __launch_bounds__(THREADS) block_copy_kernel(uint8_t* __restrict__ dst,
                                                              const uint8_t* __restrict__ src, int64_t d0,
                                                              int64_t d1, int64_t d2, int64_t s0, int64_t s1,
                                                              int64_t s2, int64_t n1, int64_t n2, int64_t items,
                                                              int64_t chunks, int64_t vecs) {
  for (int64_t item = blockIdx.x; item < items; item += gridDim.x) {
    const int64_t blk = item / chunks, chunk = item % chunks;
    const int64_t i2 = blk % n2, i1 = (blk / n2) % n1, i0 = blk / (n2 * n1);
    const uint4* from = reinterpret_cast<const uint4*>(src + i0 * s0 + i1 * s1 + i2 * s2);
    uint4* to = reinterpret_cast<uint4*>(dst + i0 * d0 + i1 * d1 + i2 * d2);
    const int64_t first = chunk * COPY_CHUNK + threadIdx.x;
    uint4 v[COPY_VECS_PER_THREAD];
#pragma unroll
    for (int j = 0; j < COPY_VECS_PER_THREAD; ++j) {
      const int64_t e = first + j * THREADS;
      if (e < vecs) v[j] = from[e];
    }
#pragma unroll
    for (int j = 0; j < COPY_VECS_PER_THREAD; ++j) {
      const int64_t e = first + j * THREADS;
      if (e < vecs) to[e] = v[j];
    }
  }
}

}  // namespace small
}  // namespace iris

using namespace iris;

extern "C" int iris_patchify(const float* x, void* out, int64_t batch, int64_t channels, int64_t height,
                             int64_t width, int64_t patch, int64_t token_start, int64_t tokens, void* stream) {
  using namespace iris::small;
  IRIS_REQUIRE(x && out, "patchify: null pointer");
  IRIS_REQUIRE(patch > 0 && height % patch == 0 && width % patch == 0 && batch >= 0 && channels > 0,
               "input is not divisible by patch_size");
  IRIS_REQUIRE(token_start >= 0 && tokens >= 0 && token_start + tokens <= (height / patch) * (width / patch),
               "patchify: token range outside the patch grid");
  IRIS_REQUIRE(channels * patch * patch < (1 << 30), "patchify: patch too large");
  const int64_t rows = batch * tokens;
  if (rows == 0) return IRIS_OK;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
  patchify_kernel<<<static_cast<unsigned>(rows < cap ? rows : cap), THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      x, reinterpret_cast<__nv_bfloat16*>(out), rows, static_cast<int>(channels), height, width,
      static_cast<int>(patch), token_start, tokens);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_unpatchify(const float* out, float* v, int64_t batch, int64_t channels, int64_t height,
                               int64_t width, int64_t patch, void* stream) {
  using namespace iris::small;
  IRIS_REQUIRE(out && v, "unpatchify: null pointer");
  IRIS_REQUIRE(patch > 0 && height % patch == 0 && width % patch == 0 && batch >= 0 && channels > 0,
               "input is not divisible by patch_size");
  const int64_t total = batch * channels * height * width;
  if (total == 0) return IRIS_OK;
  unpatchify_kernel<<<grid_for(total), THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      out, v, total, static_cast<int>(channels), height, width, static_cast<int>(patch));
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_timestep_embedding(const float* t, float* out, int64_t batch, int64_t freq_dim, float max_period,
                                       void* stream) {
  using namespace iris::small;
  IRIS_REQUIRE(t && out, "timestep_embedding: null pointer");
  IRIS_REQUIRE(freq_dim > 0 && freq_dim % 2 == 0, "freq_dim must be even");
  IRIS_REQUIRE(max_period > 0.f, "timestep_embedding: max_period must be positive");
  if (batch <= 0) return IRIS_OK;
  const int half = static_cast<int>(freq_dim / 2);
  timestep_kernel<<<grid_for(batch * half), THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      t, out, batch, half, logf(max_period));
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_gemv(const float* x, int64_t M, int64_t K, const void* w, int w_dtype, const float* bias,
                         float* out, int64_t N, int act_in, int act_out, void* stream) {
  using namespace iris::small;
  IRIS_REQUIRE(x && w && out, "gemv: null pointer");
  IRIS_REQUIRE(M > 0 && N > 0 && K > 0 && K % 8 == 0, "gemv: K must be a positive multiple of 8");
  IRIS_REQUIRE(M < (1 << 20) && N < (1ll << 31) && K < (1ll << 31), "gemv: size");
  IRIS_REQUIRE(w_dtype == IRIS_F32 || w_dtype == IRIS_BF16, "gemv: weights must be f32 or bf16");
  IRIS_REQUIRE(aligned16(x) && aligned16(w), "gemv: pointers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // two columns per warp when every warp of a full grid still gets a few groups
  const bool wide = N >= static_cast<int64_t>(num_sms()) * 4 * (THREADS / 32) * 2;
  // rows staged per pass: 2, 4 or 8 (more rows take further passes)
  const int mt = M <= 2 ? 2 : (M <= 4 ? 4 : 8);
  const int64_t smem64 = static_cast<int64_t>(mt) * K * 4;
  IRIS_REQUIRE(smem64 <= 200 * 1024, "gemv: K too large for the staged rows (K <= 6400)");
  const int smem = static_cast<int>(smem64);
  const int Mi = static_cast<int>(M), Ki = static_cast<int>(K), Ni = static_cast<int>(N);
  const int64_t per_block = static_cast<int64_t>(THREADS / 32) * (wide ? 2 : 1);
  const int64_t needed = (N + per_block - 1) / per_block;
  // the grid: the blocks resident at once (each warp then streams several
  // column groups), or fewer when there are not that many groups
#define IRIS_GEMV(TW, C, R)                                                                                          \
  {                                                                                                                  \
    auto kernel = gemv_kernel<TW, C, R>;                                                                             \
    if (smem > 48 * 1024) IRIS_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)); \
    int resident = 0;                                                                                                \
    IRIS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, kernel, THREADS, smem));                      \
    const int64_t cap = static_cast<int64_t>(num_sms()) * (resident > 0 ? resident : 1);                             \
    const unsigned grid = static_cast<unsigned>(needed < cap ? needed : cap);                                        \
    kernel<<<grid, THREADS, smem, st>>>(x, Mi, Ki, reinterpret_cast<const TW*>(w), bias, out, Ni, act_in, act_out);  \
  }
#define IRIS_GEMV_ROWS(TW, C)             \
  {                                       \
    if (mt == 2) IRIS_GEMV(TW, C, 2)      \
    else if (mt == 4) IRIS_GEMV(TW, C, 4) \
    else IRIS_GEMV(TW, C, 8)              \
  }
  if (w_dtype == IRIS_BF16) {
    if (wide) IRIS_GEMV_ROWS(__nv_bfloat16, 2) else IRIS_GEMV_ROWS(__nv_bfloat16, 1)
  } else {
    if (wide) IRIS_GEMV_ROWS(float, 2) else IRIS_GEMV_ROWS(float, 1)
  }
#undef IRIS_GEMV_ROWS
#undef IRIS_GEMV
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_add_bias_rows(const float* core, const float* bias, float* out, int64_t batch, int64_t n_blocks,
                                  int64_t width, void* stream) {
  using namespace iris::small;
  IRIS_REQUIRE(core && bias && out, "add_bias_rows: null pointer");
  const int64_t total = batch * n_blocks * width;
  if (total <= 0) return IRIS_OK;
  add_bias_rows_kernel<<<grid_for(total), THREADS, 0, static_cast<cudaStream_t>(stream)>>>(core, bias, out, batch,
                                                                                          n_blocks, width);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_cfg_euler(const float* v, const float* x, float* x_out, int64_t images, int64_t per_image,
                              float cfg_scale, float sigma, float sigma_next, int guided, void* stream) {
  using namespace iris::small;
  IRIS_REQUIRE(v && x && x_out, "cfg_euler: null pointer");
  IRIS_REQUIRE(sigma > 0.f, "cfg_euler: sigma must be positive");
  const int64_t total = images * per_image;
  if (total <= 0) return IRIS_OK;
  cfg_euler_kernel<<<grid_for(total, 4), THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      v, x, x_out, images, per_image, cfg_scale, sigma, sigma_next, guided);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_dpm_update(const float* v, const float* x, const float* x0_prev, float* x0_out, float* x_out,
                               int64_t images, int64_t per_image, float cfg_scale, int guided, float sigma,
                               int predict_x, float a, float b, float c, void* stream) {
  using namespace iris::small;
  IRIS_REQUIRE(v && x && x0_out && x_out, "dpm_update: null pointer");
  IRIS_REQUIRE(images >= 0 && per_image >= 0, "dpm_update: negative size");
  IRIS_REQUIRE(c == 0.f || x0_prev != nullptr, "dpm_update: a second-order step needs the previous x0");
  const int64_t total = images * per_image;
  if (total == 0) return IRIS_OK;
  dpm_update_kernel<<<grid_for(total, 4), THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      v, x, c == 0.f ? nullptr : x0_prev, x0_out, x_out, total, cfg_scale, guided, sigma, predict_x, a, b, c);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_all_finite(const float* x, int64_t n, int* flag, void* stream) {
  using namespace iris::small;
  IRIS_REQUIRE(x && flag, "all_finite: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  set_int_kernel<<<1, 1, 0, st>>>(flag, 1);
  if (n > 0) all_finite_kernel<<<grid_for(n, 8), THREADS, 0, st>>>(x, n, flag);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_poison_on_error(float* x, int64_t n, unsigned int mask, void* stream) {
  using namespace iris::small;
  IRIS_REQUIRE(x != nullptr || n == 0, "poison_on_error: null pointer");
  IRIS_REQUIRE(n >= 0, "poison_on_error: negative size");
  if (n == 0 || mask == 0u) return IRIS_OK;
  poison_on_error_kernel<<<grid_for(n, 8), THREADS, 0, static_cast<cudaStream_t>(stream)>>>(x, n, mask);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_block_copy(void* dst, int64_t dst_stride0, int64_t dst_stride1, int64_t dst_stride2,
                               const void* src, int64_t src_stride0, int64_t src_stride1, int64_t src_stride2,
                               int64_t count0, int64_t count1, int64_t count2, int64_t block_bytes, void* stream) {
  using namespace iris::small;
  IRIS_REQUIRE(dst && src, "block_copy: null pointer");
  IRIS_REQUIRE(count0 >= 0 && count1 >= 0 && count2 >= 0 && block_bytes >= 0, "block_copy: negative size");
  IRIS_REQUIRE(aligned16(dst) && aligned16(src) && block_bytes % 16 == 0 && dst_stride0 % 16 == 0 &&
                   dst_stride1 % 16 == 0 && dst_stride2 % 16 == 0 && src_stride0 % 16 == 0 &&
                   src_stride1 % 16 == 0 && src_stride2 % 16 == 0,
               "block_copy: pointers, strides and block size must be multiples of 16 bytes");
  const int64_t blocks = count0 * count1 * count2;
  if (blocks == 0 || block_bytes == 0) return IRIS_OK;
  const int64_t vecs = block_bytes / 16;
  const int64_t chunks = (vecs + COPY_CHUNK - 1) / COPY_CHUNK;
  const int64_t items = blocks * chunks;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
  const unsigned grid = static_cast<unsigned>(items < cap ? items : cap);
  block_copy_kernel<<<grid, THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<uint8_t*>(dst), reinterpret_cast<const uint8_t*>(src), dst_stride0, dst_stride1, dst_stride2,
      src_stride0, src_stride1, src_stride2, count1, count2, items, chunks, vecs);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}
