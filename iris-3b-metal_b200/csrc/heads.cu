// Attention-input kernels (HBM-bound): per-head RMSNorm + RoPE + the
// [B, N, H, 128] -> [B, H, N, 128] transpose, src/iris_metal/kernels.py:37-84,
// 334-397; the V head transpose of src/iris_metal/model.py:247.
//
// Half a warp per token, looping over the token's 128-wide head rows: lane l
// holds elements [8l, 8l + 8) of a head = rotary pairs 4l .. 4l+3, loaded and
// stored as 16-byte vectors (bf16); a head's sum of squares is a 16-lane
// shuffle reduction. The grid is resident and strides over the tokens.
#include "common.cuh"
#include "iris_abi_internal.h"

namespace iris {
namespace heads {

constexpr int ROWS_PER_BLOCK = 16;  // half-warps per 256-thread block

template <typename T>
IRIS_DEVICE void load8(const T* p, float (&v)[8]);
template <>
IRIS_DEVICE void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
IRIS_DEVICE void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16x2(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
IRIS_DEVICE void load8<__half>(const __half* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <typename T>
IRIS_DEVICE void store8(T* p, const float (&v)[8]);
template <>
IRIS_DEVICE void store8<float>(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
template <>
IRIS_DEVICE void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(p) =
      make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}
template <>
IRIS_DEVICE void store8<__half>(__half* p, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(p) =
      make_uint4(pack_f16x2(v[0], v[1]), pack_f16x2(v[2], v[3]), pack_f16x2(v[4], v[5]), pack_f16x2(v[6], v[7]));
}

// Sum over the 16 lanes of this half-warp; the mask names only those lanes,
// so a half-warp past the end of the rows may exit without stalling its twin.
IRIS_DEVICE float half_warp_sum(float v) {
  const unsigned mask = (threadIdx.x & 16) ? 0xffff0000u : 0x0000ffffu;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(mask, v, o);
  return v;
}

// RMSNorm * gain then rotate pairs (2i, 2i+1): (a c - b s, a s + b c).
IRIS_DEVICE void norm_rope(float (&v)[8], int sub, const float* weight, const float* cs, const float* sn, float eps) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  ss = half_warp_sum(ss);
  const float inv = rsqrtf(ss * (1.f / 128.f) + eps);
  const float4 w0 = __ldg(reinterpret_cast<const float4*>(weight + sub * 8));
  const float4 w1 = __ldg(reinterpret_cast<const float4*>(weight + sub * 8 + 4));
  const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  const float4 c4 = __ldg(reinterpret_cast<const float4*>(cs + sub * 4));
  const float4 s4 = __ldg(reinterpret_cast<const float4*>(sn + sub * 4));
  const float c[4] = {c4.x, c4.y, c4.z, c4.w}, s[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = v[2 * i] * inv * w[2 * i];
    const float b = v[2 * i + 1] * inv * w[2 * i + 1];
    v[2 * i] = a * c[i] - b * s[i];
    v[2 * i + 1] = a * s[i] + b * c[i];
  }
}

// Eight elements of a row as loaded (16 bytes of bf16 / f16, 32 of f32), kept
// packed until used so a prefetched row costs few registers.
template <typename T>
struct Raw8 {
  uint4 u;
  IRIS_DEVICE void load(const T* p) { u = *reinterpret_cast<const uint4*>(p); }
  IRIS_DEVICE void unpack(float (&v)[8]) const { load8<T>(reinterpret_cast<const T*>(&u), v); }
};
template <>
struct Raw8<float> {
  float4 a, b;
  IRIS_DEVICE void load(const float* p) {
    a = *reinterpret_cast<const float4*>(p);
    b = *reinterpret_cast<const float4*>(p + 4);
  }
  IRIS_DEVICE void unpack(float (&v)[8]) const {
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
};

// RMSNorm * gain then rotary pairs with the gain and this token's cos / sin
// already in registers (lane `sub` holds pairs 4 sub .. 4 sub + 3).
IRIS_DEVICE void norm_rope_regs(float (&v)[8], const float (&w)[8], const float (&c)[4], const float (&s)[4],
                                float eps) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += v[i] * v[i];
  ss = half_warp_sum(ss);
  const float inv = rsqrtf(ss * (1.f / 128.f) + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = v[2 * i] * inv * w[2 * i];
    const float b = v[2 * i + 1] * inv * w[2 * i + 1];
    v[2 * i] = a * c[i] - b * s[i];
    v[2 * i + 1] = a * s[i] + b * c[i];
  }
}

IRIS_DEVICE void load_gain(const float* weight, int sub, float (&w)[8]) {
  const float4 w0 = __ldg(reinterpret_cast<const float4*>(weight + sub * 8));
  const float4 w1 = __ldg(reinterpret_cast<const float4*>(weight + sub * 8 + 4));
  w[0] = w0.x; w[1] = w0.y; w[2] = w0.z; w[3] = w0.w; w[4] = w1.x; w[5] = w1.y; w[6] = w1.z; w[7] = w1.w;
}

IRIS_DEVICE void load_cs(const float* cos_t, const float* sin_t, int64_t t, int sub, float (&c)[4], float (&s)[4]) {
  const float4 c4 = __ldg(reinterpret_cast<const float4*>(cos_t + t * 64 + sub * 4));
  const float4 s4 = __ldg(reinterpret_cast<const float4*>(sin_t + t * 64 + sub * 4));
  c[0] = c4.x; c[1] = c4.y; c[2] = c4.z; c[3] = c4.w;
  s[0] = s4.x; s[1] = s4.y; s[2] = s4.z; s[3] = s4.w;
}

// One half-warp per token (grid-stride over the tokens), looping over its
// heads HEADS_IN_FLIGHT at a time with all their loads issued first. The gain
// and the token's rotary row are read once into registers: read per head they
// would move more bytes through L1 than the head itself moves through HBM.
constexpr int HEADS_IN_FLIGHT = 4;

template <typename TX, typename TO>
__global__ void __launch_bounds__(ROWS_PER_BLOCK * 16, 4) qk_norm_rope_kernel(
    const TX* __restrict__ x, int64_t batch, int64_t tokens, int64_t row_stride, int64_t col_offset, int heads,
    const float* __restrict__ weight, const float* __restrict__ cos_t, const float* __restrict__ sin_t, float eps,
    TO* __restrict__ out, int64_t n_out, int64_t offset) {
  const int sub = threadIdx.x & 15;
  const int64_t total = batch * tokens;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * ROWS_PER_BLOCK;
  float w[8];
  load_gain(weight, sub, w);
  for (int64_t bn = static_cast<int64_t>(blockIdx.x) * ROWS_PER_BLOCK + (threadIdx.x >> 4); bn < total;
       bn += stride) {
    const int64_t b = bn / tokens, t = offset + bn % tokens;
    float c[4], s[4];
    load_cs(cos_t, sin_t, t, sub, c, s);
    const TX* src = x + bn * row_stride + col_offset + sub * 8;
    TO* dst = out + (b * heads * n_out + t) * 128 + sub * 8;
    for (int h0 = 0; h0 < heads; h0 += HEADS_IN_FLIGHT) {
      Raw8<TX> raw[HEADS_IN_FLIGHT];
#pragma unroll
      for (int j = 0; j < HEADS_IN_FLIGHT; ++j)
        if (h0 + j < heads) raw[j].load(src + (h0 + j) * 128);
#pragma unroll
      for (int j = 0; j < HEADS_IN_FLIGHT; ++j) {
        if (h0 + j < heads) {
          float v[8];
          raw[j].unpack(v);
          norm_rope_regs(v, w, c, s, eps);
          store8<TO>(dst + (h0 + j) * n_out * 128, v);
        }
      }
    }
  }
}

__global__ void __launch_bounds__(ROWS_PER_BLOCK * 16, 3) qkv_heads_kernel(
    const __nv_bfloat16* __restrict__ qkv, int64_t batch, int64_t tokens, int64_t row_stride, int hq, int hkv,
    const float* __restrict__ qw, const float* __restrict__ kw, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, float eps, __nv_bfloat16* __restrict__ q_out,
    __nv_bfloat16* __restrict__ k_out, __nv_bfloat16* __restrict__ v_out, int64_t n_out, int64_t n_out_kv,
    int64_t offset, bool head_major) {
  const int sub = threadIdx.x & 15;
  const int slots = hq + 2 * hkv;
  const int64_t total = batch * tokens;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * ROWS_PER_BLOCK;
  float wq[8], wk[8];
  load_gain(qw, sub, wq);
  if (hkv > 0) load_gain(kw, sub, wk);
  for (int64_t bn = static_cast<int64_t>(blockIdx.x) * ROWS_PER_BLOCK + (threadIdx.x >> 4); bn < total;
       bn += stride) {
    const int64_t b = bn / tokens, t = offset + bn % tokens;
    float c[4], s[4];
    load_cs(cos_t, sin_t, t, sub, c, s);
    const __nv_bfloat16* src = qkv + bn * row_stride + sub * 8;
    // [b, h, t] or, head-major, [h, b, t] (contiguous per-head slices for an all-to-all)
    auto at = [&](int h, int heads, int64_t len) { return ((head_major ? h * batch + b : b * heads + h) * len + t) * 128; };
    for (int s0 = 0; s0 < slots; s0 += HEADS_IN_FLIGHT) {
      Raw8<__nv_bfloat16> raw[HEADS_IN_FLIGHT];
#pragma unroll
      for (int j = 0; j < HEADS_IN_FLIGHT; ++j)
        if (s0 + j < slots) raw[j].load(src + (s0 + j) * 128);
#pragma unroll
      for (int j = 0; j < HEADS_IN_FLIGHT; ++j) {
        const int slot = s0 + j;
        if (slot >= slots) break;
        float v[8];
        raw[j].unpack(v);
        if (slot < hq) {
          norm_rope_regs(v, wq, c, s, eps);
          store8<__nv_bfloat16>(q_out + at(slot, hq, n_out) + sub * 8, v);
        } else if (slot < hq + hkv) {
          norm_rope_regs(v, wk, c, s, eps);
          store8<__nv_bfloat16>(k_out + at(slot - hq, hkv, n_out_kv) + sub * 8, v);
        } else {
          store8<__nv_bfloat16>(v_out + at(slot - hq - hkv, hkv, n_out_kv) + sub * 8, v);
        }
      }
    }
  }
}

// Grid of a grid-stride launch over `rows` half-warp items (tokens): the blocks
// that are resident at once (from the kernel's occupancy), or fewer for small inputs.
template <typename Kernel>
inline unsigned stride_grid(Kernel kernel, int64_t rows) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, ROWS_PER_BLOCK * 16, 0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int64_t blocks = (rows + ROWS_PER_BLOCK - 1) / ROWS_PER_BLOCK;
  const int64_t cap = static_cast<int64_t>(num_sms()) * per_sm;
  return static_cast<unsigned>(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

template <typename TX, typename TO>
int launch_qk(const void* x, int64_t batch, int64_t tokens, int64_t row_stride, int64_t col_offset, int heads,
              const float* w, const float* c, const float* s, float eps, void* out, int64_t n_out, int64_t offset,
              cudaStream_t st) {
  const unsigned grid = stride_grid(qk_norm_rope_kernel<TX, TO>, batch * tokens);
  qk_norm_rope_kernel<TX, TO><<<grid, ROWS_PER_BLOCK * 16, 0, st>>>(reinterpret_cast<const TX*>(x), batch, tokens,
                                                                     row_stride, col_offset, heads, w, c, s, eps,
                                                                     reinterpret_cast<TO*>(out), n_out, offset);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

}  // namespace heads
}  // namespace iris

using namespace iris;

static int elem_size(int dtype) { return dtype == IRIS_F32 ? 4 : 2; }

extern "C" int iris_qk_norm_rope(const void* x, int x_dtype, int64_t batch, int64_t tokens, int64_t row_stride,
                                 int64_t col_offset, int64_t heads, const float* weight, const float* cos,
                                 const float* sin, float eps, void* out, int out_dtype, int64_t n_out, int64_t offset,
                                 void* stream) {
  using namespace iris::heads;
  IRIS_REQUIRE(heads > 0 && col_offset >= 0 && offset >= 0, "heads must be positive and offsets nonnegative");
  IRIS_REQUIRE(x && out && weight && cos && sin, "qk_norm_rope: null pointer");
  IRIS_REQUIRE(batch >= 0 && tokens >= 0, "qk_norm_rope: negative sizes");
  IRIS_REQUIRE(col_offset + heads * 128 <= row_stride, "qk_norm_rope needs a contiguous [B, N, W] input holding the heads");
  IRIS_REQUIRE(offset + tokens <= n_out, "qk_norm_rope rotary tables or output do not cover the written rows");
  IRIS_REQUIRE(x_dtype >= IRIS_F32 && x_dtype <= IRIS_F16 && out_dtype >= IRIS_F32 && out_dtype <= IRIS_F16,
               "qk_norm_rope: bad dtype");
  IRIS_REQUIRE(aligned16(x) && aligned16(out) && aligned16(weight) && aligned16(cos) && aligned16(sin),
               "qk_norm_rope: pointers must be 16-byte aligned");
  IRIS_REQUIRE((row_stride * elem_size(x_dtype)) % 16 == 0 && (col_offset * elem_size(x_dtype)) % 16 == 0,
               "qk_norm_rope: row stride and column offset must keep 16-byte alignment");
  if (batch * tokens == 0) return IRIS_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int h = static_cast<int>(heads);
#define IRIS_QK(TX, TO) \
  return launch_qk<TX, TO>(x, batch, tokens, row_stride, col_offset, h, weight, cos, sin, eps, out, n_out, offset, st)
#define IRIS_QK_OUT(TX)                                 \
  if (out_dtype == IRIS_F32) IRIS_QK(TX, float);         \
  if (out_dtype == IRIS_BF16) IRIS_QK(TX, __nv_bfloat16); \
  IRIS_QK(TX, __half);
  if (x_dtype == IRIS_F32) {
    IRIS_QK_OUT(float)
  }
  if (x_dtype == IRIS_BF16) {
    IRIS_QK_OUT(__nv_bfloat16)
  }
  IRIS_QK_OUT(__half)
#undef IRIS_QK_OUT
#undef IRIS_QK
}

extern "C" int iris_qkv_heads(const void* qkv, int64_t batch, int64_t tokens, int64_t row_stride, int64_t heads_q,
                              int64_t heads_kv, const float* q_weight, const float* k_weight, const float* cos,
                              const float* sin, float eps, void* q_out, void* k_out, void* v_out, int64_t n_out,
                              int64_t n_out_kv, int64_t offset, int head_major, void* stream) {
  using namespace iris::heads;
  IRIS_REQUIRE(heads_q > 0 && heads_kv >= 0 && offset >= 0, "qkv_heads: bad head counts or offset");
  IRIS_REQUIRE(qkv && q_out && q_weight && cos && sin, "qkv_heads: null pointer");
  IRIS_REQUIRE(heads_kv == 0 || (k_out && v_out && k_weight), "qkv_heads: null k/v pointer");
  IRIS_REQUIRE((heads_q + 2 * heads_kv) * 128 <= row_stride && row_stride % 8 == 0, "qkv_heads: row stride");
  IRIS_REQUIRE(offset + tokens <= n_out && (heads_kv == 0 || offset + tokens <= n_out_kv),
               "qkv_heads: output does not cover the written rows");
  IRIS_REQUIRE(aligned16(qkv) && aligned16(q_out) && aligned16(cos) && aligned16(sin) && aligned16(q_weight),
               "qkv_heads: pointers must be 16-byte aligned");
  IRIS_REQUIRE(heads_kv == 0 || (aligned16(k_out) && aligned16(v_out) && aligned16(k_weight)),
               "qkv_heads: pointers must be 16-byte aligned");
  if (batch * tokens == 0) return IRIS_OK;
  const unsigned grid = stride_grid(qkv_heads_kernel, batch * tokens);
  qkv_heads_kernel<<<grid, ROWS_PER_BLOCK * 16, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv), batch, tokens, row_stride, static_cast<int>(heads_q),
      static_cast<int>(heads_kv), q_weight, k_weight, cos, sin, eps, reinterpret_cast<__nv_bfloat16*>(q_out),
      reinterpret_cast<__nv_bfloat16*>(k_out), reinterpret_cast<__nv_bfloat16*>(v_out), n_out, n_out_kv, offset,
      head_major != 0);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}
