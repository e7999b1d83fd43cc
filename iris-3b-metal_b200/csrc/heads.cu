// Attention-input kernels (HBM-bound): per-head RMSNorm + RoPE + the
// [B, N, H, 128] -> [B, H, N, 128] transpose, src/iris_metal/kernels.py:37-84,
// 334-397; the V head transpose of src/iris_metal/model.py:247.
//
// Half a warp per (batch, token, head) row of 128: lane l holds elements
// [8l, 8l + 8) = rotary pairs 4l .. 4l+3 in registers, loaded and stored as
// 16-byte vectors (bf16). The row's sum of squares is a 16-lane shuffle
// reduction. Consecutive half-warps take consecutive heads of a token, so the
// reads of a projection row are contiguous.
#include "common.cuh"
#include "iris_abi_internal.h"

namespace iris {
namespace heads {

constexpr int ROWS_PER_BLOCK = 16;  // 256 threads

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

template <typename TX, typename TO>
__global__ void __launch_bounds__(ROWS_PER_BLOCK * 16) qk_norm_rope_kernel(
    const TX* __restrict__ x, int64_t batch, int64_t tokens, int64_t row_stride, int64_t col_offset, int heads,
    const float* __restrict__ weight, const float* __restrict__ cos_t, const float* __restrict__ sin_t, float eps,
    TO* __restrict__ out, int64_t n_out, int64_t offset) {
  const int sub = threadIdx.x & 15;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * ROWS_PER_BLOCK + (threadIdx.x >> 4);
  const int64_t total = batch * tokens * heads;
  // the whole half-warp shares `row`, so the shuffle partners stay in step
  if (row >= total) return;
  const int h = static_cast<int>(row % heads);
  const int64_t bn = row / heads;
  const int64_t b = bn / tokens, n = bn % tokens;
  float v[8];
  load8<TX>(x + bn * row_stride + col_offset + h * 128 + sub * 8, v);
  const int64_t t = offset + n;
  norm_rope(v, sub, weight, cos_t + t * 64, sin_t + t * 64, eps);
  store8<TO>(out + ((b * heads + h) * n_out + t) * 128 + sub * 8, v);
}

__global__ void __launch_bounds__(ROWS_PER_BLOCK * 16) qkv_heads_kernel(
    const __nv_bfloat16* __restrict__ qkv, int64_t batch, int64_t tokens, int64_t row_stride, int hq, int hkv,
    const float* __restrict__ qw, const float* __restrict__ kw, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, float eps, __nv_bfloat16* __restrict__ q_out,
    __nv_bfloat16* __restrict__ k_out, __nv_bfloat16* __restrict__ v_out, int64_t n_out, int64_t n_out_kv,
    int64_t offset, bool head_major) {
  const int sub = threadIdx.x & 15;
  const int slots = hq + 2 * hkv;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * ROWS_PER_BLOCK + (threadIdx.x >> 4);
  if (row >= batch * tokens * slots) return;
  const int slot = static_cast<int>(row % slots);
  const int64_t bn = row / slots;
  const int64_t b = bn / tokens, n = bn % tokens;
  const int64_t t = offset + n;
  float v[8];
  load8<__nv_bfloat16>(qkv + bn * row_stride + slot * 128 + sub * 8, v);
  // [b, h, t] or, head-major, [h, b, t] (contiguous per-head slices for an all-to-all)
  auto at = [&](int h, int heads, int64_t len) { return (head_major ? h * batch + b : b * heads + h) * len + t; };
  if (slot < hq) {
    norm_rope(v, sub, qw, cos_t + t * 64, sin_t + t * 64, eps);
    store8<__nv_bfloat16>(q_out + at(slot, hq, n_out) * 128 + sub * 8, v);
  } else if (slot < hq + hkv) {
    const int h = slot - hq;
    norm_rope(v, sub, kw, cos_t + t * 64, sin_t + t * 64, eps);
    store8<__nv_bfloat16>(k_out + at(h, hkv, n_out_kv) * 128 + sub * 8, v);
  } else {
    const int h = slot - hq - hkv;
    store8<__nv_bfloat16>(v_out + at(h, hkv, n_out_kv) * 128 + sub * 8, v);
  }
}

template <typename TX, typename TO>
int launch_qk(const void* x, int64_t batch, int64_t tokens, int64_t row_stride, int64_t col_offset, int heads,
              const float* w, const float* c, const float* s, float eps, void* out, int64_t n_out, int64_t offset,
              cudaStream_t st) {
  const int64_t rows = batch * tokens * heads;
  const unsigned grid = static_cast<unsigned>((rows + ROWS_PER_BLOCK - 1) / ROWS_PER_BLOCK);
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
  const int64_t rows = batch * tokens * (heads_q + 2 * heads_kv);
  const unsigned grid = static_cast<unsigned>((rows + ROWS_PER_BLOCK - 1) / ROWS_PER_BLOCK);
  qkv_heads_kernel<<<grid, ROWS_PER_BLOCK * 16, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv), batch, tokens, row_stride, static_cast<int>(heads_q),
      static_cast<int>(heads_kv), q_weight, k_weight, cos, sin, eps, reinterpret_cast<__nv_bfloat16*>(q_out),
      reinterpret_cast<__nv_bfloat16*>(k_out), reinterpret_cast<__nv_bfloat16*>(v_out), n_out, n_out_kv, offset,
      head_major != 0);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}
