// Row kernels on the 3072-wide residual stream (HBM-bound):
//   rms_norm_modulate           src/iris_metal/kernels.py:116-146, 413-452
//   gated_residual_rms_norm(+)  src/iris_metal/kernels.py:148-175, 455-480
//   rms_norm_add_rows           TextEmbedder norm + position table
//
// Rows whose width is a multiple of 512 (3072 here) take one 128-thread CTA
// each (see gated_residual_row_kernel); other widths one warp per row, where
// lane l owns the 4-element vectors l, l + 32, ... so every
// warp load is one coalesced 512-byte (fp32) or 256-byte (bf16) segment. The
// whole row stays in registers (NV vectors per lane, width = 128 * NV), so
// each row is read once and written once; the sum of squares is a warp
// shuffle reduction.
#include <algorithm>

#include "common.cuh"
#include "iris_abi_internal.h"

namespace iris {
namespace rows {

constexpr int WARPS = 8;  // rows per 256-thread block

template <typename T>
struct Vec4 {};
template <>
struct Vec4<float> {
  IRIS_DEVICE static float4 load(const float* p) { return *reinterpret_cast<const float4*>(p); }
  IRIS_DEVICE static void store(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
};
template <>
struct Vec4<__nv_bfloat16> {
  IRIS_DEVICE static float4 load(const __nv_bfloat16* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
    return make_float4(a.x, a.y, b.x, b.y);
  }
  IRIS_DEVICE static void store(__nv_bfloat16* p, float4 v) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
};
template <>
struct Vec4<__half> {
  IRIS_DEVICE static float4 load(const __half* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  IRIS_DEVICE static void store(__half* p, float4 v) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_f16x2(v.x, v.y), pack_f16x2(v.z, v.w));
  }
};

IRIS_DEVICE float4 ld4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
IRIS_DEVICE float sumsq(float4 v) { return v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w; }

template <typename TX, typename TO, int NV>
__global__ void __launch_bounds__(WARPS * 32) rms_norm_modulate_kernel(
    const TX* __restrict__ x, RowMap xmap, TO* __restrict__ out, const float* __restrict__ weight,
    const float* __restrict__ shift, const float* __restrict__ scale, int64_t mod_stride, int64_t rows,
    int64_t rows_per_batch, int width, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * WARPS + (threadIdx.x >> 5);
  if (r >= rows) return;
  const TX* xr = x + xmap(r) * width;
  const int nv = width >> 7;
  float4 v[NV];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (i < nv) {
      v[i] = Vec4<TX>::load(xr + (i * 32 + lane) * 4);
      ss += sumsq(v[i]);
    }
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / static_cast<float>(width) + eps);
  const int64_t b = r / rows_per_batch;
  const float* sh = shift + b * mod_stride;
  const float* sc = scale + b * mod_stride;
  TO* o = out + r * width;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (i < nv) {
      const int e = (i * 32 + lane) * 4;
      const float4 w = ld4(weight + e), s4 = ld4(sh + e), c4 = ld4(sc + e);
      float4 h;
      h.x = v[i].x * inv * w.x * (1.f + c4.x) + s4.x;
      h.y = v[i].y * inv * w.y * (1.f + c4.y) + s4.y;
      h.z = v[i].z * inv * w.z * (1.f + c4.z) + s4.z;
      h.w = v[i].w * inv * w.w * (1.f + c4.w) + s4.w;
      Vec4<TO>::store(o + e, h);
    }
  }
}

// residual[r] += gate[b] * rms_norm(branch[r]) * weight; then optionally the
// next branch input from the updated row (norm+modulate or silu(t + x)).
template <typename TB, typename TO, int NV>
__global__ void __launch_bounds__(WARPS * 32) gated_residual_kernel(
    float* __restrict__ residual, RowMap rmap, const TB* __restrict__ branch, RowMap bmap,
    const float* __restrict__ weight, const float* __restrict__ gate, int64_t mod_stride, int64_t rows,
    int64_t rows_per_batch, int width, float eps, int next_mode, const float* __restrict__ next_weight,
    const float* __restrict__ next_shift, const float* __restrict__ next_scale, int64_t next_mod_stride,
    TO* __restrict__ next_out, RowMap nmap) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * WARPS + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int nv = width >> 7;
  const TB* br = branch + bmap(r) * width;
  float* xr = residual + rmap(r) * width;
  float4 v[NV];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (i < nv) {
      v[i] = Vec4<TB>::load(br + (i * 32 + lane) * 4);
      ss += sumsq(v[i]);
    }
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / static_cast<float>(width) + eps);
  const int64_t b = r / rows_per_batch;
  const float* g = gate + b * mod_stride;
  float ss2 = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (i < nv) {
      const int e = (i * 32 + lane) * 4;
      const float4 w = ld4(weight + e), g4 = ld4(g + e);
      float4 x = *reinterpret_cast<const float4*>(xr + e);
      x.x += g4.x * (v[i].x * inv * w.x);
      x.y += g4.y * (v[i].y * inv * w.y);
      x.z += g4.z * (v[i].z * inv * w.z);
      x.w += g4.w * (v[i].w * inv * w.w);
      *reinterpret_cast<float4*>(xr + e) = x;
      v[i] = x;
      ss2 += sumsq(x);
    }
  }
  if (next_mode == IRIS_NEXT_NONE) return;
  TO* o = next_out + nmap(r) * width;
  const float* sh = next_shift + b * next_mod_stride;
  if (next_mode == IRIS_NEXT_NORM_MODULATE) {
    ss2 = warp_sum(ss2);
    const float inv2 = rsqrtf(ss2 / static_cast<float>(width) + eps);
    const float* sc = next_scale + b * next_mod_stride;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (i < nv) {
        const int e = (i * 32 + lane) * 4;
        const float4 w = ld4(next_weight + e), s4 = ld4(sh + e), c4 = ld4(sc + e);
        float4 h;
        h.x = v[i].x * inv2 * w.x * (1.f + c4.x) + s4.x;
        h.y = v[i].y * inv2 * w.y * (1.f + c4.y) + s4.y;
        h.z = v[i].z * inv2 * w.z * (1.f + c4.z) + s4.z;
        h.w = v[i].w * inv2 * w.w * (1.f + c4.w) + s4.w;
        Vec4<TO>::store(o + e, h);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (i < nv) {
        const int e = (i * 32 + lane) * 4;
        const float4 t4 = ld4(sh + e);
        float4 h;
        const float a0 = t4.x + v[i].x, a1 = t4.y + v[i].y, a2 = t4.z + v[i].z, a3 = t4.w + v[i].w;
        h.x = a0 / (1.f + __expf(-a0));
        h.y = a1 / (1.f + __expf(-a1));
        h.z = a2 / (1.f + __expf(-a2));
        h.w = a3 / (1.f + __expf(-a3));
        Vec4<TO>::store(o + e, h);
      }
    }
  }
}

// The same update with one 128-thread CTA per row (widths that are a multiple
// of 512: thread t owns the 4-vectors t, t + 128, ...). Few registers per
// thread keep up to 16 rows per SM in flight, which the warp-per-row form
// cannot at 3072 columns; sums are reduced across the 4 warps in shared memory.
constexpr int ROW_THREADS = 128;

IRIS_DEVICE float block_sum(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  return red[0] + red[1] + red[2] + red[3];
}

// 16 bytes of a row as loaded (8 bf16 / f16 or 4 f32 elements), kept packed
// until used so that a prefetched row costs few registers.
template <typename T>
struct Raw16 {
  static constexpr int E = 8;
  uint4 u;
  IRIS_DEVICE void load(const T* p) { u = *reinterpret_cast<const uint4*>(p); }
  IRIS_DEVICE float4 lo() const { return Vec4<T>::load(reinterpret_cast<const T*>(&u)); }
  IRIS_DEVICE float4 hi() const { return Vec4<T>::load(reinterpret_cast<const T*>(&u) + 4); }
};
template <>
struct Raw16<float> {
  static constexpr int E = 4;
  float4 u;
  IRIS_DEVICE void load(const float* p) { u = *reinterpret_cast<const float4*>(p); }
  IRIS_DEVICE float4 lo() const { return u; }
  IRIS_DEVICE float4 hi() const { return u; }
};

// Stores E / 4 float4 as TO with the widest vector stores (16 bytes where the
// E outputs of 2-byte types fill one).
template <typename TO, int E>
IRIS_DEVICE void store_vec(TO* p, const float4 (&y)[E / 4]) {
  if constexpr (E == 8 && sizeof(TO) == 2) {
    uint2 a, b;
    Vec4<TO>::store(reinterpret_cast<TO*>(&a), y[0]);
    Vec4<TO>::store(reinterpret_cast<TO*>(&b), y[1]);
    *reinterpret_cast<uint4*>(p) = make_uint4(a.x, a.y, b.x, b.y);
  } else {
#pragma unroll
    for (int h = 0; h < E / 4; ++h) Vec4<TO>::store(p + 4 * h, y[h]);
  }
}

// 16-byte asynchronous copy global -> shared (cp.async, L2 only), in commit groups per thread.
IRIS_DEVICE void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem)), "l"(gmem) : "memory");
}
IRIS_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
IRIS_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Persistent form for widths of 128 * CPT columns: a resident grid of
// 128-thread CTAs strides over the rows, one row per CTA at a time; thread t
// owns the 16-byte vectors t, t + 128, ... of every row (CPT columns).
// Each thread streams its own vectors of the next RING rows into shared
// memory with cp.async while it works on the current one, so no thread waits
// on another's copies and a row's loads never wait for the block reduction of
// the row before. The per-column factors w * (1 + scale[b]) and shift[b] stay
// in registers while b is unchanged (fetched before the first row lands);
// re-reading the three fp32 parameter rows per row would move six times the
// row's bytes through L1. One barrier per row (the block-wide sum of squares,
// double-buffered). On B200 this runs the BF16 [8192, 3072] -> BF16 case at
// 0.76 of the measured HBM copy bandwidth and the FP32-input case at 0.93.
constexpr int NORM_RING = 2;

template <typename TX, typename TO, int CPT>
__global__ void __launch_bounds__(ROW_THREADS, CPT <= 24 ? 4 : 3) rms_norm_modulate_row_kernel(
    const TX* __restrict__ x, RowMap xmap, TO* __restrict__ out, const float* __restrict__ weight,
    const float* __restrict__ shift, const float* __restrict__ scale, int64_t mod_stride, int64_t rows,
    int64_t rows_per_batch, float eps) {
  constexpr int E = Raw16<TX>::E;  // elements per 16-byte vector
  constexpr int VPT = CPT / E;     // vectors per thread per row
  constexpr int WIDTH = CPT * ROW_THREADS;
  extern __shared__ __align__(16) uint4 ring[];  // [NORM_RING][VPT][ROW_THREADS]
  __shared__ float red[2][ROW_THREADS / 32];
  const int t = threadIdx.x;
  const int64_t G = gridDim.x;
  // identity row maps (the common case) skip the map's 64-bit divisions
  const bool ident = xmap.seg_stride == 0 && xmap.seg_offset == 0 && xmap.seg_rows >= rows;
  auto issue = [&](int64_t r, int slot) {
    const TX* src = x + (ident ? r : xmap(r)) * WIDTH;
#pragma unroll
    for (int i = 0; i < VPT; ++i) cp_async16(&ring[(slot * VPT + i) * ROW_THREADS + t], src + (i * ROW_THREADS + t) * E);
  };
#pragma unroll
  for (int k = 0; k < NORM_RING; ++k) {
    const int64_t r = blockIdx.x + k * G;
    if (r < rows) issue(r, k);
    cp_async_commit();  // one group per slot, empty past the last row, so the wait counts stay fixed
  }
  float mul[CPT], add[CPT];
  int64_t cur_b = -1, b_end = 0;  // rows [.., b_end) belong to batch cur_b; rows only grow
  auto load_mods = [&](int64_t b) {
    const float* sh = shift + b * mod_stride;
    const float* sc = scale + b * mod_stride;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
#pragma unroll
      for (int h = 0; h < E / 4; ++h) {
        const int e = (i * ROW_THREADS + t) * E + 4 * h, j = i * E + 4 * h;
        const float4 g = ld4(weight + e), c = ld4(sc + e), a = ld4(sh + e);
        mul[j] = g.x * (1.f + c.x);
        mul[j + 1] = g.y * (1.f + c.y);
        mul[j + 2] = g.z * (1.f + c.z);
        mul[j + 3] = g.w * (1.f + c.w);
        add[j] = a.x;
        add[j + 1] = a.y;
        add[j + 2] = a.z;
        add[j + 3] = a.w;
      }
    }
  };
  if (static_cast<int64_t>(blockIdx.x) < rows) {
    cur_b = blockIdx.x / rows_per_batch;
    b_end = (cur_b + 1) * rows_per_batch;
    load_mods(cur_b);
  }
  int it = 0;
  for (int64_t r = blockIdx.x; r < rows; r += G, ++it) {
    const int slot = it % NORM_RING;
    cp_async_wait<NORM_RING - 1>();
    Raw16<TX> v[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) v[i].u = *reinterpret_cast<const decltype(v[i].u)*>(&ring[(slot * VPT + i) * ROW_THREADS + t]);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) ss += E == 8 ? sumsq(v[i].lo()) + sumsq(v[i].hi()) : sumsq(v[i].lo());
    // the slot's values are in registers (ss depends on all of them): refill it
    const int64_t rn = r + NORM_RING * G;
    if (rn < rows) {
      asm volatile("" ::"f"(ss));
      issue(rn, slot);
    }
    cp_async_commit();
    ss = warp_sum(ss);
    if ((t & 31) == 0) red[it & 1][t >> 5] = ss;
    __syncthreads();  // red[it & 1] is rewritten two rows later, after the next barrier
    const float inv = rsqrtf((red[it & 1][0] + red[it & 1][1] + red[it & 1][2] + red[it & 1][3]) / WIDTH + eps);
    if (r >= b_end) {
      cur_b = r / rows_per_batch;
      b_end = (cur_b + 1) * rows_per_batch;
      load_mods(cur_b);
    }
    TO* o = out + r * WIDTH;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float4 y[E / 4];
#pragma unroll
      for (int h = 0; h < E / 4; ++h) {
        const float4 xv = h == 0 ? v[i].lo() : v[i].hi();
        const int j = i * E + 4 * h;
        y[h] = make_float4(xv.x * inv * mul[j] + add[j], xv.y * inv * mul[j + 1] + add[j + 1],
                           xv.z * inv * mul[j + 2] + add[j + 2], xv.w * inv * mul[j + 3] + add[j + 3]);
      }
      store_vec<TO, E>(o + (i * ROW_THREADS + t) * E, y);
    }
  }
  cp_async_wait<0>();
}

// One residual update of the row kernel: the arguments of
// iris_gated_residual_rms_norm for one stream's rows.
struct ResidualSeg {
  float* residual;
  RowMap rmap;
  const void* branch;
  RowMap bmap;
  const float* weight;
  const float* gate;
  int64_t mod_stride, rows, rows_per_batch;
  int next_mode;
  const float* next_weight;
  const float* next_shift;
  const float* next_scale;
  int64_t next_mod_stride;
  void* next_out;
  RowMap nmap;
};

// Up to two segments (a dual block's text and image rows) in one launch: CTA
// r < seg[0].rows takes row r of segment 0, the others row r - seg[0].rows of
// segment 1.
struct ResidualRows {
  ResidualSeg seg[2];
  int count;
};

template <typename TB, typename TO, int VPT>
__global__ void __launch_bounds__(ROW_THREADS) gated_residual_row_kernel(const __grid_constant__ ResidualRows rr,
                                                                         int width, float eps) {
  __shared__ float red[2][4];
  const bool second = rr.count > 1 && static_cast<int64_t>(blockIdx.x) >= rr.seg[0].rows;
  const ResidualSeg& sg = rr.seg[second ? 1 : 0];
  const int64_t r = static_cast<int64_t>(blockIdx.x) - (second ? rr.seg[0].rows : 0);
  float* __restrict__ residual = sg.residual;
  const RowMap rmap = sg.rmap, bmap = sg.bmap, nmap = sg.nmap;
  const TB* __restrict__ branch = reinterpret_cast<const TB*>(sg.branch);
  const float* __restrict__ weight = sg.weight;
  const float* __restrict__ gate = sg.gate;
  const int64_t mod_stride = sg.mod_stride, rows_per_batch = sg.rows_per_batch;
  const int next_mode = sg.next_mode;
  const float* __restrict__ next_weight = sg.next_weight;
  const float* __restrict__ next_shift = sg.next_shift;
  const float* __restrict__ next_scale = sg.next_scale;
  const int64_t next_mod_stride = sg.next_mod_stride;
  TO* __restrict__ next_out = reinterpret_cast<TO*>(sg.next_out);
  const int t = threadIdx.x;
  const TB* br = branch + bmap(r) * width;
  float* xr = residual + rmap(r) * width;
  float4 v[VPT], x[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int e = (i * ROW_THREADS + t) * 4;
    v[i] = Vec4<TB>::load(br + e);
    x[i] = *reinterpret_cast<const float4*>(xr + e);
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) ss += sumsq(v[i]);
  const float inv = rsqrtf(block_sum(ss, red[0]) / static_cast<float>(width) + eps);
  const int64_t b = r / rows_per_batch;
  const float* g = gate + b * mod_stride;
  float ss2 = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int e = (i * ROW_THREADS + t) * 4;
    const float4 w = ld4(weight + e), g4 = ld4(g + e);
    x[i].x += g4.x * (v[i].x * inv * w.x);
    x[i].y += g4.y * (v[i].y * inv * w.y);
    x[i].z += g4.z * (v[i].z * inv * w.z);
    x[i].w += g4.w * (v[i].w * inv * w.w);
    *reinterpret_cast<float4*>(xr + e) = x[i];
    ss2 += sumsq(x[i]);
  }
  if (next_mode == IRIS_NEXT_NONE) return;
  TO* o = next_out + nmap(r) * width;
  const float* sh = next_shift + b * next_mod_stride;
  if (next_mode == IRIS_NEXT_NORM_MODULATE) {
    const float inv2 = rsqrtf(block_sum(ss2, red[1]) / static_cast<float>(width) + eps);
    const float* sc = next_scale + b * next_mod_stride;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int e = (i * ROW_THREADS + t) * 4;
      const float4 w = ld4(next_weight + e), s4 = ld4(sh + e), c4 = ld4(sc + e);
      float4 h;
      h.x = x[i].x * inv2 * w.x * (1.f + c4.x) + s4.x;
      h.y = x[i].y * inv2 * w.y * (1.f + c4.y) + s4.y;
      h.z = x[i].z * inv2 * w.z * (1.f + c4.z) + s4.z;
      h.w = x[i].w * inv2 * w.w * (1.f + c4.w) + s4.w;
      Vec4<TO>::store(o + e, h);
    }
  } else {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int e = (i * ROW_THREADS + t) * 4;
      const float4 t4 = ld4(sh + e);
      const float a0 = t4.x + x[i].x, a1 = t4.y + x[i].y, a2 = t4.z + x[i].z, a3 = t4.w + x[i].w;
      float4 h;
      h.x = a0 / (1.f + __expf(-a0));
      h.y = a1 / (1.f + __expf(-a1));
      h.z = a2 / (1.f + __expf(-a2));
      h.w = a3 / (1.f + __expf(-a3));
      Vec4<TO>::store(o + e, h);
    }
  }
}

template <int NV>
__global__ void __launch_bounds__(WARPS * 32) rms_norm_add_kernel(float* __restrict__ x,
                                                                   const float* __restrict__ weight,
                                                                   const float* __restrict__ add, int64_t rows,
                                                                   int64_t rows_per_batch, int width, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * WARPS + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int nv = width >> 7;
  float* xr = x + r * width;
  const float* ar = add + (r % rows_per_batch) * width;
  float4 v[NV];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (i < nv) {
      v[i] = *reinterpret_cast<const float4*>(xr + (i * 32 + lane) * 4);
      ss += sumsq(v[i]);
    }
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / static_cast<float>(width) + eps);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (i < nv) {
      const int e = (i * 32 + lane) * 4;
      const float4 w = ld4(weight + e), a = ld4(ar + e);
      float4 h;
      h.x = w.x * (v[i].x * inv) + a.x;
      h.y = w.y * (v[i].y * inv) + a.y;
      h.z = w.z * (v[i].z * inv) + a.z;
      h.w = w.w * (v[i].w * inv) + a.w;
      *reinterpret_cast<float4*>(xr + e) = h;
    }
  }
}

// NV buckets: a row of width 128 * nv runs with the smallest bucket >= nv.
#define IRIS_NV_DISPATCH(nv, MACRO) \
  if ((nv) <= 2) {                  \
    MACRO(2);                       \
  } else if ((nv) <= 4) {           \
    MACRO(4);                       \
  } else if ((nv) <= 8) {           \
    MACRO(8);                       \
  } else if ((nv) <= 16) {          \
    MACRO(16);                      \
  } else if ((nv) <= 24) {          \
    MACRO(24);                      \
  } else {                          \
    MACRO(32);                      \
  }

// CTAs of a persistent row launch: as many as are resident at once, at most one per row.
template <typename Kernel>
unsigned resident_grid(Kernel kernel, int64_t rows, int smem = 0) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, ROW_THREADS, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int64_t cap = static_cast<int64_t>(num_sms()) * per_sm;
  return static_cast<unsigned>(rows < cap ? (rows > 0 ? rows : 1) : cap);
}

template <typename TX, typename TO>
int launch_norm_modulate(const void* x, RowMap xm, void* out, const float* w, const float* sh, const float* sc,
                         int64_t mod_stride, int64_t rows, int64_t rpb, int width, float eps, cudaStream_t st) {
  constexpr int E = Raw16<TX>::E;
  const int cpt = width / ROW_THREADS;
  if (width % (E * ROW_THREADS) == 0 && (cpt == 8 || cpt == 16 || cpt == 24 || cpt == 32) && aligned16(x) &&
      aligned16(sh) && aligned16(sc)) {
    const int smem = NORM_RING * width * static_cast<int>(sizeof(TX));
#define IRIS_ROW(CPT)                                                                                              \
  {                                                                                                                \
    auto kernel = rms_norm_modulate_row_kernel<TX, TO, CPT>;                                                       \
    if (smem > 48 * 1024) IRIS_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)); \
    const unsigned grid = resident_grid(kernel, rows, smem);                                                       \
    kernel<<<grid, ROW_THREADS, smem, st>>>(reinterpret_cast<const TX*>(x), xm, reinterpret_cast<TO*>(out), w, sh, \
                                            sc, mod_stride, rows, rpb, eps);                                      \
  }
    switch (cpt) {
      case 8: IRIS_ROW(8); break;
      case 16: IRIS_ROW(16); break;
      case 24: IRIS_ROW(24); break;
      default: IRIS_ROW(32); break;
    }
#undef IRIS_ROW
    IRIS_CUDA(cudaGetLastError());
    return IRIS_OK;
  }
  const int nv = width / 128;
  const unsigned grid = static_cast<unsigned>((rows + WARPS - 1) / WARPS);
#define IRIS_LAUNCH(NV)                                                                                           \
  rms_norm_modulate_kernel<TX, TO, NV><<<grid, WARPS * 32, 0, st>>>(reinterpret_cast<const TX*>(x), xm,          \
                                                                     reinterpret_cast<TO*>(out), w, sh, sc,      \
                                                                     mod_stride, rows, rpb, width, eps)
  IRIS_NV_DISPATCH(nv, IRIS_LAUNCH)
#undef IRIS_LAUNCH
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

bool row_kernel_width(int width) { return width % (4 * ROW_THREADS) == 0 && width / (4 * ROW_THREADS) <= 8; }

// The row kernel over one or two segments (all rows of one width, branch and
// next-output dtypes).
template <typename TB, typename TO>
int launch_residual_rows(const ResidualRows& rr, int width, float eps, cudaStream_t st) {
  const int64_t rows = rr.seg[0].rows + (rr.count > 1 ? rr.seg[1].rows : 0);
  if (rows == 0) return IRIS_OK;
  IRIS_REQUIRE(rows < (1ll << 31), "gated_residual_rms_norm_: too many rows");
  const int vpt = width / (4 * ROW_THREADS);
#define IRIS_ROW(VPT) \
  gated_residual_row_kernel<TB, TO, VPT><<<static_cast<unsigned>(rows), ROW_THREADS, 0, st>>>(rr, width, eps)
  switch (vpt) {
    case 1: IRIS_ROW(1); break;
    case 2: IRIS_ROW(2); break;
    case 3: IRIS_ROW(3); break;
    case 4: IRIS_ROW(4); break;
    case 5: IRIS_ROW(5); break;
    case 6: IRIS_ROW(6); break;
    case 7: IRIS_ROW(7); break;
    default: IRIS_ROW(8); break;
  }
#undef IRIS_ROW
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

template <typename TB, typename TO>
int launch_residual(float* res, RowMap rm, const void* branch, RowMap bm, const float* w, const float* gate,
                    int64_t ms, int64_t rows, int64_t rpb, int width, float eps, int mode, const float* nw,
                    const float* nsh, const float* nsc, int64_t nms, void* nout, RowMap nm, cudaStream_t st) {
  if (row_kernel_width(width) && rows < (1ll << 31)) {
    ResidualRows rr{};
    rr.count = 1;
    rr.seg[0] = ResidualSeg{res, rm, branch, bm, w, gate, ms, rows, rpb, mode, nw, nsh, nsc, nms, nout, nm};
    return launch_residual_rows<TB, TO>(rr, width, eps, st);
  }
  const int nv = width / 128;
  const unsigned grid = static_cast<unsigned>((rows + WARPS - 1) / WARPS);
#define IRIS_LAUNCH(NV)                                                                                            \
  gated_residual_kernel<TB, TO, NV><<<grid, WARPS * 32, 0, st>>>(res, rm, reinterpret_cast<const TB*>(branch), bm, \
                                                                  w, gate, ms, rows, rpb, width, eps, mode, nw, nsh,  \
                                                                  nsc, nms, reinterpret_cast<TO*>(nout), nm)
  IRIS_NV_DISPATCH(nv, IRIS_LAUNCH)
#undef IRIS_LAUNCH
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

}  // namespace rows
}  // namespace iris

using namespace iris;

static int check_mod(const float* p, int64_t stride, const char* name) {
  if (p == nullptr) return set_error(IRIS_EINVAL, "%s: null modulation pointer", name);
  if (!aligned16(p) || stride % 4 != 0)
    return set_error(IRIS_EINVAL, "%s: modulation rows must be 16-byte aligned (stride %% 4 == 0)", name);
  return IRIS_OK;
}

extern "C" int iris_rms_norm_modulate(const void* x, int x_dtype, int64_t x_seg_rows, int64_t x_seg_stride,
                                      int64_t x_seg_offset, void* out, int out_dtype, const float* weight,
                                      const float* shift, const float* scale, int64_t mod_stride, int64_t rows,
                                      int64_t rows_per_batch, int64_t width, float eps, void* stream) {
  using namespace iris::rows;
  IRIS_REQUIRE(x && out && weight, "rms_norm_modulate: null pointer");
  IRIS_REQUIRE(width > 0 && width % 128 == 0 && width <= 4096,
               "rms_norm_modulate needs a contiguous input, width % 128 == 0 (and <= 4096)");
  IRIS_REQUIRE(rows >= 0 && rows_per_batch > 0 && x_seg_rows > 0, "rms_norm_modulate: bad row counts");
  IRIS_REQUIRE(x_dtype == IRIS_F32 || x_dtype == IRIS_BF16, "rms_norm_modulate: x must be f32 or bf16");
  IRIS_REQUIRE(out_dtype >= IRIS_F32 && out_dtype <= IRIS_F16, "rms_norm_modulate: bad out dtype");
  IRIS_REQUIRE(aligned16(x) && aligned16(out) && aligned16(weight), "rms_norm_modulate: pointers must be 16-byte aligned");
  IRIS_CHECK_STATUS(check_mod(shift, mod_stride, "rms_norm_modulate"));
  IRIS_CHECK_STATUS(check_mod(scale, mod_stride, "rms_norm_modulate"));
  if (rows == 0) return IRIS_OK;
  const RowMap xm{x_seg_rows, x_seg_stride, x_seg_offset};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int w = static_cast<int>(width);
  if (x_dtype == IRIS_F32) {
    if (out_dtype == IRIS_BF16)
      return launch_norm_modulate<float, __nv_bfloat16>(x, xm, out, weight, shift, scale, mod_stride, rows,
                                                        rows_per_batch, w, eps, st);
    if (out_dtype == IRIS_F16)
      return launch_norm_modulate<float, __half>(x, xm, out, weight, shift, scale, mod_stride, rows, rows_per_batch,
                                                 w, eps, st);
    return launch_norm_modulate<float, float>(x, xm, out, weight, shift, scale, mod_stride, rows, rows_per_batch, w,
                                              eps, st);
  }
  if (out_dtype == IRIS_BF16)
    return launch_norm_modulate<__nv_bfloat16, __nv_bfloat16>(x, xm, out, weight, shift, scale, mod_stride, rows,
                                                              rows_per_batch, w, eps, st);
  if (out_dtype == IRIS_F16)
    return launch_norm_modulate<__nv_bfloat16, __half>(x, xm, out, weight, shift, scale, mod_stride, rows,
                                                       rows_per_batch, w, eps, st);
  return launch_norm_modulate<__nv_bfloat16, float>(x, xm, out, weight, shift, scale, mod_stride, rows,
                                                    rows_per_batch, w, eps, st);
}

static int check_residual(const iris_residual_problem& q, int branch_dtype, int next_out_dtype, int64_t width) {
  IRIS_REQUIRE(q.residual && q.branch && q.weight, "gated_residual_rms_norm_: null pointer");
  IRIS_REQUIRE(width > 0 && width % 128 == 0 && width <= 4096, "gated_residual_rms_norm_: width % 128 != 0");
  IRIS_REQUIRE(q.rows >= 0 && q.rows_per_batch > 0 && q.res_seg_rows > 0 && q.br_seg_rows > 0,
               "gated_residual_rms_norm_: bad row counts");
  IRIS_REQUIRE(branch_dtype >= IRIS_F32 && branch_dtype <= IRIS_F16, "gated_residual_rms_norm_: bad branch dtype");
  IRIS_REQUIRE(aligned16(q.residual) && aligned16(q.branch) && aligned16(q.weight),
               "gated_residual_rms_norm_: pointers must be 16-byte aligned");
  IRIS_CHECK_STATUS(check_mod(q.gate, q.mod_stride, "gated_residual_rms_norm_"));
  IRIS_REQUIRE(q.next_mode >= IRIS_NEXT_NONE && q.next_mode <= IRIS_NEXT_SILU_ADD,
               "gated_residual_rms_norm_: bad next_mode");
  if (q.next_mode != IRIS_NEXT_NONE) {
    IRIS_REQUIRE(q.next_out && aligned16(q.next_out), "gated_residual_rms_norm_: next output must be 16-byte aligned");
    IRIS_REQUIRE(next_out_dtype == IRIS_BF16 || next_out_dtype == IRIS_F32, "gated_residual_rms_norm_: next dtype");
    IRIS_REQUIRE(q.nx_seg_rows > 0, "gated_residual_rms_norm_: next row map needs seg_rows > 0");
    IRIS_CHECK_STATUS(check_mod(q.next_shift, q.next_mod_stride, "gated_residual_rms_norm_ (next)"));
    if (q.next_mode == IRIS_NEXT_NORM_MODULATE) {
      IRIS_REQUIRE(q.next_weight && aligned16(q.next_weight), "gated_residual_rms_norm_: next weight");
      IRIS_CHECK_STATUS(check_mod(q.next_scale, q.next_mod_stride, "gated_residual_rms_norm_ (next)"));
    }
  }
  return IRIS_OK;
}

template <typename TB, typename TO>
static int residual_problems(const iris_residual_problem* qs, int count, int64_t width, float eps, cudaStream_t st) {
  using namespace iris::rows;
  const int w = static_cast<int>(width);
  auto seg = [](const iris_residual_problem& q) {
    return ResidualSeg{q.residual, RowMap{q.res_seg_rows, q.res_seg_stride, q.res_seg_offset}, q.branch,
                       RowMap{q.br_seg_rows, q.br_seg_stride, q.br_seg_offset}, q.weight, q.gate, q.mod_stride, q.rows,
                       q.rows_per_batch, q.next_mode, q.next_weight, q.next_shift, q.next_scale, q.next_mod_stride,
                       q.next_out, RowMap{q.nx_seg_rows > 0 ? q.nx_seg_rows : 1, q.nx_seg_stride, q.nx_seg_offset}};
  };
  if (row_kernel_width(w)) {
    ResidualRows rr{};
    rr.count = count;
    for (int i = 0; i < count; ++i) rr.seg[i] = seg(qs[i]);
    return launch_residual_rows<TB, TO>(rr, w, eps, st);
  }
  for (int i = 0; i < count; ++i) {
    const ResidualSeg g = seg(qs[i]);
    if (g.rows == 0) continue;
    const int status = launch_residual<TB, TO>(g.residual, g.rmap, g.branch, g.bmap, g.weight, g.gate, g.mod_stride,
                                               g.rows, g.rows_per_batch, w, eps, g.next_mode, g.next_weight,
                                               g.next_shift, g.next_scale, g.next_mod_stride, g.next_out, g.nmap, st);
    if (status != IRIS_OK) return status;
  }
  return IRIS_OK;
}

extern "C" int iris_gated_residual_rms_norm_grouped(const iris_residual_problem* problems, int count,
                                                    int branch_dtype, int next_out_dtype, int64_t width, float eps,
                                                    void* stream) {
  IRIS_REQUIRE(problems != nullptr && count >= 1 && count <= 2, "gated_residual_rms_norm_: 1 or 2 problems per launch");
  for (int i = 0; i < count; ++i) IRIS_CHECK_STATUS(check_residual(problems[i], branch_dtype, next_out_dtype, width));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool nf32 = next_out_dtype == IRIS_F32;
#define IRIS_RES(TB, TO) return residual_problems<TB, TO>(problems, count, width, eps, st)
  if (branch_dtype == IRIS_BF16) {
    if (nf32) IRIS_RES(__nv_bfloat16, float);
    IRIS_RES(__nv_bfloat16, __nv_bfloat16);
  }
  if (branch_dtype == IRIS_F16) {
    if (nf32) IRIS_RES(__half, float);
    IRIS_RES(__half, __nv_bfloat16);
  }
  if (nf32) IRIS_RES(float, float);
  IRIS_RES(float, __nv_bfloat16);
#undef IRIS_RES
}

extern "C" int iris_gated_residual_rms_norm(float* residual, int64_t res_seg_rows, int64_t res_seg_stride,
                                            int64_t res_seg_offset, const void* branch, int branch_dtype,
                                            int64_t br_seg_rows, int64_t br_seg_stride, int64_t br_seg_offset,
                                            const float* weight, const float* gate, int64_t mod_stride, int64_t rows,
                                            int64_t rows_per_batch, int64_t width, float eps, int next_mode,
                                            const float* next_weight, const float* next_shift,
                                            const float* next_scale, int64_t next_mod_stride, void* next_out,
                                            int next_out_dtype, int64_t nx_seg_rows, int64_t nx_seg_stride,
                                            int64_t nx_seg_offset, void* stream) {
  const iris_residual_problem q{residual,    res_seg_rows,    res_seg_stride, res_seg_offset, branch,
                                br_seg_rows, br_seg_stride,   br_seg_offset,  weight,         gate,
                                mod_stride,  rows,            rows_per_batch, next_mode,      next_weight,
                                next_shift,  next_scale,      next_mod_stride, next_out,      nx_seg_rows,
                                nx_seg_stride, nx_seg_offset};
  return iris_gated_residual_rms_norm_grouped(&q, 1, branch_dtype, next_out_dtype, width, eps, stream);
}

extern "C" int iris_rms_norm_add_rows(float* x, const float* weight, const float* add, int64_t rows,
                                      int64_t rows_per_batch, int64_t width, float eps, void* stream) {
  using namespace iris::rows;
  IRIS_REQUIRE(x && weight && add, "rms_norm_add_rows: null pointer");
  IRIS_REQUIRE(width > 0 && width % 128 == 0 && width <= 4096, "rms_norm_add_rows: width % 128 != 0");
  IRIS_REQUIRE(rows >= 0 && rows_per_batch > 0, "rms_norm_add_rows: bad row counts");
  IRIS_REQUIRE(aligned16(x) && aligned16(weight) && aligned16(add), "rms_norm_add_rows: alignment");
  if (rows == 0) return IRIS_OK;
  const int nv = static_cast<int>(width / 128);
  const unsigned grid = static_cast<unsigned>((rows + WARPS - 1) / WARPS);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define IRIS_LAUNCH(NV) \
  rms_norm_add_kernel<NV><<<grid, WARPS * 32, 0, st>>>(x, weight, add, rows, rows_per_batch, static_cast<int>(width), eps)
  IRIS_NV_DISPATCH(nv, IRIS_LAUNCH)
#undef IRIS_LAUNCH
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}
