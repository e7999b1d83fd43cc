// Kernels of the text adapters that run once per prompt before sampling:
// LayerwiseTextEmbedder ("lap_blocks2") and TransformerTextEmbedder
// ("blocks2"), src/iris3b/nn/embeddings.py:79-266. Their linears run on the
// tensor-core GEMM (iris_gemm_bf16 with the ADD / SILU / SWIGLU epilogues) and
// their norms on iris_rms_norm_modulate; what is left is here:
//
//   small_attention   softmax(q k^T / sqrt(d)) v over short sequences read
//                     straight from a [rows, 3 * heads * d] q | k | v
//                     projection: the encoder layers of one token (12 keys,
//                     d = 80, no QK norm) or the text tokens of one prompt
//                     (300 keys, d = 128, per-head QK RMSNorm, pad keys masked
//                     except on the diagonal: embeddings.py:151-162,199-205)
//   layer_pool        Linear(layers -> 1) over the layer axis (embeddings.py:262-264)
//
// The attention is SIMT: at these sizes (<= 1.1 GFLOP per prompt, under 1% of
// the adapter's GEMM work) a tensor-core tile would be mostly padding.
#include "common.cuh"
#include "iris_abi_internal.h"

namespace iris {
namespace adapter {

constexpr int THREADS = 128;
constexpr int WARPS = THREADS / 32;
constexpr int QBLOCK = 64;  // queries per CTA
constexpr int MAX_HEAD_DIM = 128;

// One CTA per (sequence, head, block of 64 queries). The sequence's keys
// (QK-normed when k_gain is given, rounded to bf16) and values are staged in
// shared memory: keys with a row stride of d + 2 elements, so the 32 lanes of
// a warp, each scoring its own key, read 32 different banks. Each warp then
// takes one query at a time: the query row (normed, scaled by
// log2(e) / sqrt(d)) in shared memory, lane l scores keys l, l + 32, ...,
// online softmax across rounds of 32 keys, and lane l accumulates output
// dimensions l, l + 32, ... of sum_j p_j v_j.
__global__ void __launch_bounds__(THREADS) small_attention_kernel(
    const __nv_bfloat16* __restrict__ qkv, int64_t row_stride, int n, int heads, int hd, int qblocks,
    const float* __restrict__ q_gain, const float* __restrict__ k_gain, float eps, const uint8_t* __restrict__ key_mask,
    float scale_log2, __nv_bfloat16* __restrict__ out, int64_t out_stride) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int kstride = hd + 2;
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* vs = ks + static_cast<size_t>(n) * kstride;
  float* qs = reinterpret_cast<float*>(vs + static_cast<size_t>(n) * hd + ((n * hd) & 1));

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int item = blockIdx.x;
  const int qb = item % qblocks;
  const int h = (item / qblocks) % heads;
  const int64_t seq = item / (static_cast<int64_t>(qblocks) * heads);
  const __nv_bfloat16* rows = qkv + seq * n * row_stride;
  const int qcol = h * hd, kcol = (heads + h) * hd, vcol = (2 * heads + h) * hd;
  const int pairs = hd / 2;

  // stage keys and values: one warp per row, lane p handles element pairs p, p + 32
  for (int j = warp; j < n; j += WARPS) {
    const __nv_bfloat16* kr = rows + static_cast<int64_t>(j) * row_stride + kcol;
    const __nv_bfloat16* vr = rows + static_cast<int64_t>(j) * row_stride + vcol;
    float2 kv[2];
    float ss = 0.f;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int p = lane + 32 * t;
      kv[t] = make_float2(0.f, 0.f);
      if (p < pairs) {
        kv[t] = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(kr + 2 * p));
        ss = fmaf(kv[t].x, kv[t].x, fmaf(kv[t].y, kv[t].y, ss));
        *reinterpret_cast<uint32_t*>(vs + j * hd + 2 * p) = *reinterpret_cast<const uint32_t*>(vr + 2 * p);
      }
    }
    float inv = 1.f;
    if (k_gain != nullptr) inv = rsqrtf(warp_sum(ss) / static_cast<float>(hd) + eps);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int p = lane + 32 * t;
      if (p < pairs) {
        float a = kv[t].x, b = kv[t].y;
        if (k_gain != nullptr) {
          a *= inv * __ldg(k_gain + 2 * p);
          b *= inv * __ldg(k_gain + 2 * p + 1);
        }
        *reinterpret_cast<uint32_t*>(ks + j * kstride + 2 * p) = pack_bf16x2(a, b);
      }
    }
  }
  __syncthreads();

  float* q = qs + warp * MAX_HEAD_DIM;
  const int q_end = min(n, (qb + 1) * QBLOCK);
  for (int i = qb * QBLOCK + warp; i < q_end; i += WARPS) {
    const __nv_bfloat16* qr = rows + static_cast<int64_t>(i) * row_stride + qcol;
    float2 qv[2];
    float ss = 0.f;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int p = lane + 32 * t;
      qv[t] = make_float2(0.f, 0.f);
      if (p < pairs) {
        qv[t] = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(qr + 2 * p));
        ss = fmaf(qv[t].x, qv[t].x, fmaf(qv[t].y, qv[t].y, ss));
      }
    }
    float inv = scale_log2;
    if (q_gain != nullptr) inv *= rsqrtf(warp_sum(ss) / static_cast<float>(hd) + eps);
    __syncwarp();  // the previous query's readers are done with q
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int p = lane + 32 * t;
      if (p < pairs) {
        const float ga = q_gain != nullptr ? __ldg(q_gain + 2 * p) : 1.f;
        const float gb = q_gain != nullptr ? __ldg(q_gain + 2 * p + 1) : 1.f;
        q[2 * p] = qv[t].x * inv * ga;
        q[2 * p + 1] = qv[t].y * inv * gb;
      }
    }
    __syncwarp();

    float m = -INFINITY, l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int r0 = 0; r0 < n; r0 += 32) {
      const int j = r0 + lane;
      float s = -INFINITY;
      if (j < n && (key_mask == nullptr || key_mask[seq * n + j] != 0 || j == i)) {
        const uint32_t* kr = reinterpret_cast<const uint32_t*>(ks + j * kstride);
        float dot = 0.f;
        for (int p = 0; p < pairs; ++p) {
          const float2 kk = unpack_bf16x2(kr[p]);
          dot = fmaf(q[2 * p], kk.x, fmaf(q[2 * p + 1], kk.y, dot));
        }
        s = dot;
      }
      float mc = s;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, o));
      const float m_new = fmaxf(m, mc);
      if (m_new == -INFINITY) continue;  // every key so far masked (the diagonal comes later)
      const float p = s == -INFINITY ? 0.f : exp2f(s - m_new);
      const float alpha = m == -INFINITY ? 0.f : exp2f(m - m_new);
      l = l * alpha + warp_sum(p);
#pragma unroll
      for (int t = 0; t < 4; ++t) acc[t] *= alpha;
      const int cnt = min(32, n - r0);
      for (int jj = 0; jj < cnt; ++jj) {
        const float pj = __shfl_sync(0xffffffffu, p, jj);
        const __nv_bfloat16* vr = vs + (r0 + jj) * hd;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int d = lane + 32 * t;
          if (d < hd) acc[t] = fmaf(pj, bf16_to_f32(vr[d]), acc[t]);
        }
      }
      m = m_new;
    }
    const float rl = 1.f / l;  // l > 0: every query attends at least itself
    __nv_bfloat16* orow = out + (seq * n + i) * out_stride + static_cast<int64_t>(h) * hd;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int d = lane + 32 * t;
      if (d < hd) orow[d] = __float2bfloat16_rn(acc[t] * rl);
    }
  }
}

// out[r, c] = sum_l w[l] x[r * layers + l, c] + bias (bf16 out), 4 columns per thread.
__global__ void layer_pool_kernel(const float* __restrict__ x, int64_t rows, int layers, int64_t width,
                                  const float* __restrict__ w, const float* __restrict__ bias,
                                  __nv_bfloat16* __restrict__ out) {
  const int64_t vecs = width / 4;
  const float b = __ldg(bias);
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < rows * vecs;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = e / vecs, c = (e % vecs) * 4;
    float4 s = make_float4(b, b, b, b);
    for (int l = 0; l < layers; ++l) {
      const float wl = __ldg(w + l);
      const float4 v = *reinterpret_cast<const float4*>(x + (r * layers + l) * width + c);
      s.x = fmaf(wl, v.x, s.x);
      s.y = fmaf(wl, v.y, s.y);
      s.z = fmaf(wl, v.z, s.z);
      s.w = fmaf(wl, v.w, s.w);
    }
    uint2 packed = make_uint2(pack_bf16x2(s.x, s.y), pack_bf16x2(s.z, s.w));
    *reinterpret_cast<uint2*>(out + r * width + c) = packed;
  }
}

inline size_t attention_smem(int64_t n, int64_t hd) {
  const int64_t kv = n * (hd + 2) + n * hd + ((n * hd) & 1);
  return static_cast<size_t>(kv * 2 + WARPS * MAX_HEAD_DIM * 4);
}

}  // namespace adapter
}  // namespace iris

using namespace iris;

extern "C" int iris_small_attention(const void* qkv, int64_t seqs, int64_t n, int64_t heads, int64_t head_dim,
                                    int64_t row_stride, const float* q_gain, const float* k_gain, float eps,
                                    const uint8_t* key_mask, float scale, void* out, int64_t out_stride,
                                    void* stream) {
  using namespace iris::adapter;
  IRIS_REQUIRE(qkv && out, "small_attention: null pointer");
  IRIS_REQUIRE((q_gain == nullptr) == (k_gain == nullptr), "small_attention: give both QK-norm gains or neither");
  IRIS_REQUIRE(seqs >= 0 && n > 0 && heads > 0, "small_attention: empty shape");
  IRIS_REQUIRE(head_dim > 0 && head_dim <= MAX_HEAD_DIM && head_dim % 8 == 0,
               "small_attention: head_dim must be a multiple of 8 up to 128");
  IRIS_REQUIRE(row_stride >= 3 * heads * head_dim && row_stride % 8 == 0 && out_stride >= heads * head_dim &&
                   out_stride % 2 == 0,
               "small_attention: row strides");
  IRIS_REQUIRE(aligned16(qkv) && aligned_n(out, 4), "small_attention: qkv must be 16-byte aligned, out 4-byte");
  IRIS_REQUIRE(q_gain == nullptr || (aligned16(q_gain) && aligned16(k_gain)), "small_attention: gains alignment");
  const size_t smem = attention_smem(n, head_dim);
  IRIS_REQUIRE(smem <= 227 * 1024, "small_attention: the sequence's keys and values must fit in shared memory "
                                   "(n * (4 head_dim + 4) bytes <= 227 KB)");
  if (seqs == 0) return IRIS_OK;
  const int64_t qblocks = (n + QBLOCK - 1) / QBLOCK;
  const int64_t items = seqs * heads * qblocks;
  IRIS_REQUIRE(items < (1ll << 31), "small_attention: too many sequences");
  if (smem > 48 * 1024)
    IRIS_CUDA(cudaFuncSetAttribute(small_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(smem)));
  const float scale_log2 = scale * 1.4426950408889634f;
  small_attention_kernel<<<static_cast<unsigned>(items), THREADS, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(qkv), row_stride, static_cast<int>(n), static_cast<int>(heads),
      static_cast<int>(head_dim), static_cast<int>(qblocks), q_gain, k_gain, eps, key_mask, scale_log2,
      static_cast<__nv_bfloat16*>(out), out_stride);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_layer_pool(const float* x, int64_t rows, int64_t layers, int64_t width, const float* weight,
                               const float* bias, void* out, void* stream) {
  using namespace iris::adapter;
  IRIS_REQUIRE(x && weight && bias && out, "layer_pool: null pointer");
  IRIS_REQUIRE(rows >= 0 && layers > 0 && width > 0 && width % 4 == 0, "layer_pool: width must be a multiple of 4");
  IRIS_REQUIRE(aligned16(x) && aligned_n(out, 8), "layer_pool: x must be 16-byte aligned, out 8-byte");
  if (rows == 0) return IRIS_OK;
  const int64_t total = rows * (width / 4);
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  layer_pool_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, rows, static_cast<int>(layers), width, weight, bias, static_cast<__nv_bfloat16*>(out));
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}
