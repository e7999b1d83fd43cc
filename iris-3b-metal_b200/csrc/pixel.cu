// Pixel-stage kernels, one thread per pixel with its 16 channels in
// registers (HBM-bound; the 16 -> 64 -> 16 MLP weights sit in shared memory):
//   pixel_rms_norm    src/iris_metal/kernels.py:217-232, 486-498
//   pixel_mlp_        src/iris_metal/kernels.py:235-293, 527-584 (post-mod PiT
//                     tail, src/iris3b/models/blocks/pit.py:88-92)
//   pixel_mlp_head    the last block's tail fused with FinalLayer + fold
//                     (src/iris3b/models/dit.py:53-62, 367-374)
//   pixel_embed       PixelEmbedder (src/iris3b/nn/embeddings.py:319-328)
//                     fused with the first block's pixel_rms_norm.
// With bf16 pixels the kernel rounds where the reference's autocast path
// materialises bf16 values; with an fp32 pixel stream it rounds nothing.
#include "common.cuh"
#include "iris_abi_internal.h"

namespace iris {
namespace pixel {

constexpr int C = 16;
constexpr int HID = 64;
// RGB, plus the extra input channel of the depth fine-tune's widened embedders
// (src/iris3b/downstream/depth.py:30-38)
constexpr int MAX_IN_CHANNELS = 4;
constexpr int THREADS = 256;

IRIS_DEVICE void load16(const void* p, int64_t i, bool f32, float (&x)[C]) {
  if (f32) {
    const float4* q = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i * C);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 v = q[j];
      x[4 * j] = v.x; x[4 * j + 1] = v.y; x[4 * j + 2] = v.z; x[4 * j + 3] = v.w;
    }
  } else {
    const uint4* q = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p) + i * C);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint4 u = q[j];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = unpack_bf16x2(w[h]);
        x[8 * j + 2 * h] = f.x;
        x[8 * j + 2 * h + 1] = f.y;
      }
    }
  }
}

IRIS_DEVICE void store16(void* p, int64_t i, bool f32, const float (&x)[C]) {
  if (f32) {
    float4* q = reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i * C);
#pragma unroll
    for (int j = 0; j < 4; ++j) q[j] = make_float4(x[4 * j], x[4 * j + 1], x[4 * j + 2], x[4 * j + 3]);
  } else {
    uint4* q = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p) + i * C);
#pragma unroll
    for (int j = 0; j < 2; ++j)
      q[j] = make_uint4(pack_bf16x2(x[8 * j], x[8 * j + 1]), pack_bf16x2(x[8 * j + 2], x[8 * j + 3]),
                        pack_bf16x2(x[8 * j + 4], x[8 * j + 5]), pack_bf16x2(x[8 * j + 6], x[8 * j + 7]));
  }
}

IRIS_DEVICE float inv_rms16(const float (&x)[C], float eps) {
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < C; ++c) ss += x[c] * x[c];
  return rsqrtf(ss / C + eps);
}

// GELU(a) = a Phi(a) (the exact, erf form) with erf from Abramowitz & Stegun
// 7.1.26 (|error| <= 1.5e-7 in erf): for x = |a| / sqrt(2),
// 1 - erf(x) = t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-x^2), t = 1 / (1 + p x),
// and Phi(a) = 1 - q for a >= 0, q for a < 0, with q = (1 - erf(x)) / 2. One
// reciprocal and one exponential on the MUFU, the rest on the FMA pipe: about
// half the instructions of erff, whose results it matches to about 1e-6
// relative (the bf16 roundings downstream flip in rare ties only).
IRIS_DEVICE float gelu_erf(float a) {
  const float x = fabsf(a) * 0.70710678118654752f;
  const float t = __fdividef(1.f, fmaf(0.3275911f, x, 1.f));
  float poly = fmaf(t, 1.061405429f, -1.453152027f);
  poly = fmaf(t, poly, 1.421413741f);
  poly = fmaf(t, poly, -0.284496736f);
  poly = fmaf(t, poly, 0.254829592f);
  const float q = 0.5f * t * poly * __expf(-x * x);
  return a * (a >= 0.f ? 1.f - q : q);
}

struct MlpWeights {
  float w1[HID * C];  // [64, 16]
  float b1[HID];
  float w2[C * HID];  // [16, 64]
  float b2[C];
  float nw[C];
  float nnw[C];
  float fw[3 * C];
  float fb[4];
};

IRIS_DEVICE void load_weights(MlpWeights& s, const __nv_bfloat16* w1, const __nv_bfloat16* b1,
                              const __nv_bfloat16* w2, const __nv_bfloat16* b2, const float* nw, const float* nnw,
                              const float* fw, const float* fb) {
  for (int i = threadIdx.x; i < HID * C; i += blockDim.x) {
    s.w1[i] = __bfloat162float(w1[i]);
    s.w2[i] = __bfloat162float(w2[i]);
  }
  for (int i = threadIdx.x; i < HID; i += blockDim.x) s.b1[i] = __bfloat162float(b1[i]);
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    s.b2[i] = __bfloat162float(b2[i]);
    s.nw[i] = nw[i];
    s.nnw[i] = nnw ? nnw[i] : 0.f;
  }
  if (fw != nullptr) {
    for (int i = threadIdx.x; i < 3 * C; i += blockDim.x) s.fw[i] = fw[i];
    for (int i = threadIdx.x; i < 3; i += blockDim.x) s.fb[i] = fb[i];
  }
  __syncthreads();
}

// The post-modulated PiT tail for one pixel; returns the updated stream in x.
template <bool ROUND>
IRIS_DEVICE void pit_tail(float (&x)[C], const float (&attn)[C], const __nv_bfloat16* mod, const MlpWeights& s,
                          float eps) {
  auto r = [](float v) { return ROUND ? round_bf16(v) : v; };
  float m[4 * C];
  {
    const uint4* q = reinterpret_cast<const uint4*>(mod);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint4 u = q[j];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = unpack_bf16x2(w[h]);
        m[8 * j + 2 * h] = f.x;
        m[8 * j + 2 * h + 1] = f.y;
      }
    }
  }
#pragma unroll
  for (int c = 0; c < C; ++c) x[c] = r(x[c] + r(attn[c] * (1.f + m[c]) + m[C + c]));
  const float inv = inv_rms16(x, eps);
  float h[C];
#pragma unroll
  for (int c = 0; c < C; ++c) h[c] = r(x[c] * inv * s.nw[c]);
  float out[C];
#pragma unroll
  for (int c = 0; c < C; ++c) out[c] = s.b2[c];
#pragma unroll 4
  for (int j = 0; j < HID; ++j) {
    float a = s.b1[j];
#pragma unroll
    for (int c = 0; c < C; ++c) a = fmaf(h[c], s.w1[j * C + c], a);
    const float g = r(gelu_erf(r(a)));
#pragma unroll
    for (int c = 0; c < C; ++c) out[c] = fmaf(g, s.w2[c * HID + j], out[c]);
  }
#pragma unroll
  for (int c = 0; c < C; ++c) x[c] = r(x[c] + r(r(out[c]) * (1.f + m[2 * C + c]) + m[3 * C + c]));
}

// gelu_erf on a pair, the polynomial and products on packed f32x2 instructions
IRIS_DEVICE float2 gelu_erf2(float2 a) {
  const float2 x = __fmul2_rn(make_float2(fabsf(a.x), fabsf(a.y)), make_float2(0.70710678118654752f, 0.70710678118654752f));
  const float2 d = __ffma2_rn(x, make_float2(0.3275911f, 0.3275911f), make_float2(1.f, 1.f));
  const float2 t = make_float2(__fdividef(1.f, d.x), __fdividef(1.f, d.y));
  // half the published coefficients: q = (1 - erf(x)) / 2 directly
  float2 poly = __ffma2_rn(t, make_float2(0.5307027145f, 0.5307027145f), make_float2(-0.7265760135f, -0.7265760135f));
  poly = __ffma2_rn(t, poly, make_float2(0.7107068705f, 0.7107068705f));
  poly = __ffma2_rn(t, poly, make_float2(-0.142248368f, -0.142248368f));
  poly = __ffma2_rn(t, poly, make_float2(0.127414796f, 0.127414796f));
  const float2 x2 = __fmul2_rn(x, x);
  const float2 e = make_float2(__expf(-x2.x), __expf(-x2.y));
  const float2 q = __fmul2_rn(__fmul2_rn(t, poly), e);
  return make_float2(a.x * (a.x >= 0.f ? 1.f - q.x : q.x), a.y * (a.y >= 0.f ? 1.f - q.y : q.y));
}

// ---------------------------------------------------------------------------
// Tensor-core form of the pixel tail: one warp per 16-pixel tile. The MLP
// (16 -> 64 -> 16) runs as mma.sync m16n8k16 BF16 -> FP32 (8 MMAs each way);
// fc1's accumulator fragments are, after bias + GELU, exactly fc2's A
// fragments. Every per-pixel elementwise step happens in the fragment layout:
// lane = 4 g + c holds pixels g and g + 8 of the tile and its fragment slots
// j = 0..3. The MMAs' channel axis (fc1's k, fc2's n) is permuted so that slot
// j is channel 4c + j: a lane's four channels of a pixel are contiguous, one
// 8-byte (bf16) or 16-byte (fp32) access each, and a warp's access covers
// whole sectors. 16-channel sums reduce over the lane quad.
IRIS_DEVICE void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

IRIS_DEVICE float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  return v;
}

IRIS_DEVICE uint32_t ld_bf16x2(const __nv_bfloat16* p) { return *reinterpret_cast<const uint32_t*>(p); }

// the channel behind the MMAs' logical channel index k (0..15): the lane quad
// position c = (k % 8) / 2 and slot j = k % 2 + 2 (k / 8) hold channel 4c + j
IRIS_DEVICE int frag_channel(int k) { return 4 * ((k & 7) >> 1) + (k & 1) + 2 * (k >> 3); }

// A tile's inputs for this lane (fragment layout: pixels g and g + 8, channels
// 4c .. 4c + 3): the pixels, the attention branch and the four modulation
// vectors (scale1, shift1, scale2, shift2), as bf16 pairs (slots 0-1, 2-3).
struct TileIn {
  float p[2][4];
  uint32_t at[2][2];
  uint32_t m[2][4][2];  // [half][scale1, shift1, scale2, shift2][slot pair]
};

constexpr int MMA_THREADS = 128;  // 4 warps per block
// Each warp streams its tiles' inputs through a ring of MMA_RING shared-memory
// slots with cp.async (16-byte pieces, whole sectors), so MMA_RING - 1 tiles'
// loads are in flight while one computes, without holding registers. A slot:
// the tile's pixels (fp32 or bf16), its attention branch, and its modulation
// rows padded to 144 bytes (conflict-free 8-byte reads by the fragment layout).
constexpr int MMA_RING = 4;
constexpr int MOD_ROW_BYTES = 4 * C * 2 + 16;
__host__ __device__ constexpr int mma_slot_bytes(bool f32) { return 16 * C * (f32 ? 4 : 2) + 16 * C * 2 + 16 * MOD_ROW_BYTES; }
__host__ __device__ constexpr int mma_smem_bytes(bool f32) { return (MMA_THREADS / 32) * MMA_RING * mma_slot_bytes(f32); }
constexpr int MMA_BLOCKS_PER_SM = 3;  // 168 registers a thread

IRIS_DEVICE void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem)), "l"(gmem) : "memory");
}
IRIS_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
IRIS_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <bool F32, bool HEAD>
__global__ void __launch_bounds__(MMA_THREADS, MMA_BLOCKS_PER_SM) pixel_mlp_mma_kernel(
    void* pixels, const __nv_bfloat16* __restrict__ branch, const __nv_bfloat16* __restrict__ mods,
    const float* __restrict__ nw, const __nv_bfloat16* __restrict__ w1, const __nv_bfloat16* __restrict__ b1,
    const __nv_bfloat16* __restrict__ w2, const __nv_bfloat16* __restrict__ b2, const float* __restrict__ nnw,
    __nv_bfloat16* __restrict__ next_input, const float* __restrict__ fw, const float* __restrict__ fb,
    float* __restrict__ v, int64_t n, int64_t height, int64_t width, int patch, int64_t token_start,
    int64_t tokens, float eps) {
  constexpr bool ROUND = !F32;
  auto r = [](float x) { return ROUND ? round_bf16(x) : x; };
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  // B fragments of W1^T (k = in channel, n = hidden) and W2^T (k = hidden, n = out channel)
  uint32_t bw1[8][2], bw2[4][2][2];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {  // logical k (2c, 2c+1) and (2c+8, 2c+9) = channels 4c .. 4c + 3
    const __nv_bfloat16* row = w1 + (nt * 8 + g) * C;
    bw1[nt][0] = ld_bf16x2(row + 4 * c);
    bw1[nt][1] = ld_bf16x2(row + 4 * c + 2);
  }
#pragma unroll
  for (int ks = 0; ks < 4; ++ks)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const __nv_bfloat16* row = w2 + frag_channel(nt * 8 + g) * HID + ks * 16;  // logical output n
      bw2[ks][nt][0] = ld_bf16x2(row + 2 * c);
      bw2[ks][nt][1] = ld_bf16x2(row + 2 * c + 8);
    }
  float bias1[8][2], bias2[4], gain[4], gain_next[4];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    bias1[nt][0] = __bfloat162float(b1[nt * 8 + 2 * c]);
    bias1[nt][1] = __bfloat162float(b1[nt * 8 + 2 * c + 1]);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int ch = 4 * c + j;
    bias2[j] = __bfloat162float(b2[ch]);
    gain[j] = nw[ch];
    gain_next[j] = nnw[ch];
  }
  const int pp = patch * patch;
  const int64_t gw = width / patch;
  const int64_t tiles = n / 16;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);

  // this warp's ring of tile slots
  extern __shared__ __align__(16) uint8_t pix_smem[];
  uint8_t* ring = pix_smem + (threadIdx.x >> 5) * MMA_RING * mma_slot_bytes(F32);
  constexpr int PIX_BYTES = 16 * C * (F32 ? 4 : 2);
  // the tile's inputs into slot `slot`: pixels, branch, modulation (three
  // contiguous runs of global memory), 16-byte pieces spread over the lanes
  auto issue_tile = [&](int64_t tile, int slot) {
    uint8_t* dst = ring + slot * mma_slot_bytes(F32);
    const uint8_t* px_src = reinterpret_cast<const uint8_t*>(pixels) + tile * PIX_BYTES;
    const uint8_t* br_src = reinterpret_cast<const uint8_t*>(branch + tile * 16 * C);
    const uint8_t* md_src = reinterpret_cast<const uint8_t*>(mods + tile * 16 * 4 * C);
#pragma unroll
    for (int e = lane; e < PIX_BYTES / 16; e += 32) cp_async16(dst + e * 16, px_src + e * 16);
    cp_async16(dst + PIX_BYTES + lane * 16, br_src + lane * 16);  // 512 bytes: one piece per lane
#pragma unroll
    for (int e = lane; e < 16 * 8; e += 32)  // 16 pixels x 8 pieces of 16 bytes
      cp_async16(dst + PIX_BYTES + 512 + (e >> 3) * MOD_ROW_BYTES + (e & 7) * 16, md_src + e * 16);
  };
  // this lane's fragment of the tile in `slot` (pixels g and g + 8, channels 4c .. 4c + 3)
  auto read_tile = [&](int slot, TileIn& in) {
    const uint8_t* src = ring + slot * mma_slot_bytes(F32);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int px = g + 8 * half;
      if (F32) {
        const float4 pv = *reinterpret_cast<const float4*>(src + (px * C + 4 * c) * 4);
        in.p[half][0] = pv.x;
        in.p[half][1] = pv.y;
        in.p[half][2] = pv.z;
        in.p[half][3] = pv.w;
      } else {
        const uint2 pv = *reinterpret_cast<const uint2*>(src + (px * C + 4 * c) * 2);
        const float2 lo = unpack_bf16x2(pv.x), hi = unpack_bf16x2(pv.y);
        in.p[half][0] = lo.x;
        in.p[half][1] = lo.y;
        in.p[half][2] = hi.x;
        in.p[half][3] = hi.y;
      }
      const uint2 at = *reinterpret_cast<const uint2*>(src + PIX_BYTES + (px * C + 4 * c) * 2);
      in.at[half][0] = at.x;
      in.at[half][1] = at.y;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint2 mv = *reinterpret_cast<const uint2*>(src + PIX_BYTES + 512 + px * MOD_ROW_BYTES + (k * C + 4 * c) * 2);
        in.m[half][k][0] = mv.x;
        in.m[half][k][1] = mv.y;
      }
    }
  };

  // where the head's tile lands in v: all 16 pixels lie in one patch (patch^2 % 16 == 0),
  // so the patch's position is worked out once per tile
  struct Fold {
    int64_t base, plane;
    int k0;
  };
  auto fold_of = [&](int64_t tile) {
    Fold f;
    const int64_t p0 = tile * 16;
    const int64_t patch_idx = p0 / pp;
    f.k0 = static_cast<int>(p0 - patch_idx * pp);
    const int64_t bb = patch_idx / tokens;
    const int64_t l = token_start + (patch_idx - bb * tokens);
    const int64_t gy = l / gw;
    f.plane = height * width;
    f.base = bb * 3 * f.plane + gy * patch * width + (l - gy * gw) * patch;
    return f;
  };

  auto process = [&](int64_t tile, const TileIn& in) {
    Fold fold = {0, 0, 0};
    if (HEAD) fold = fold_of(tile);
    float x[2][4], h[2][4];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {  // slot pairs (0, 1) and (2, 3): channels 4c + 2jj, + 1
        const float2 at = unpack_bf16x2(in.at[half][jj]);
        const float2 s1 = unpack_bf16x2(in.m[half][0][jj]);
        const float2 t1 = unpack_bf16x2(in.m[half][1][jj]);
        x[half][2 * jj] = r(in.p[half][2 * jj] + r(at.x * (1.f + s1.x) + t1.x));
        x[half][2 * jj + 1] = r(in.p[half][2 * jj + 1] + r(at.y * (1.f + s1.y) + t1.y));
      }
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) ss += x[half][j] * x[half][j];
      const float inv = rsqrtf(quad_sum(ss) / C + eps);
#pragma unroll
      for (int j = 0; j < 4; ++j) h[half][j] = x[half][j] * inv * gain[j];
    }
    // A fragment of the normed pixels (bf16)
    const uint32_t a[4] = {pack_bf16x2(h[0][0], h[0][1]), pack_bf16x2(h[1][0], h[1][1]),
                           pack_bf16x2(h[0][2], h[0][3]), pack_bf16x2(h[1][2], h[1][3])};
    uint32_t ga[4][4];  // fc2 A fragments: GELU(fc1) in bf16
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      mma_bf16_16816(acc, a, bw1[nt][0], bw1[nt][1]);
      float gl[4];
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        const float2 gv = gelu_erf2(make_float2(r(acc[j] + bias1[nt][0]), r(acc[j + 1] + bias1[nt][1])));
        gl[j] = gv.x;
        gl[j + 1] = gv.y;
      }
      const int ks = nt >> 1, hi = nt & 1;
      ga[ks][2 * hi] = pack_bf16x2(gl[0], gl[1]);      // row g
      ga[ks][2 * hi + 1] = pack_bf16x2(gl[2], gl[3]);  // row g + 8
    }
    float out[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) mma_bf16_16816(acc, ga[ks], bw2[ks][nt][0], bw2[ks][nt][1]);
      // acc: logical outputs (g, 8nt + 2c + e) and (g + 8, ...) = channel 4c + 2nt + e -> slot 2nt + e
      out[0][2 * nt] = acc[0];
      out[0][2 * nt + 1] = acc[1];
      out[1][2 * nt] = acc[2];
      out[1][2 * nt + 1] = acc[3];
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int64_t px = tile * 16 + g + 8 * half;
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const float2 s2 = unpack_bf16x2(in.m[half][2][jj]);
        const float2 t2 = unpack_bf16x2(in.m[half][3][jj]);
        const float m0 = r(out[half][2 * jj] + bias2[2 * jj]), m1 = r(out[half][2 * jj + 1] + bias2[2 * jj + 1]);
        x[half][2 * jj] = r(x[half][2 * jj] + r(m0 * (1.f + s2.x) + t2.x));
        x[half][2 * jj + 1] = r(x[half][2 * jj + 1] + r(m1 * (1.f + s2.y) + t2.y));
      }
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) ss += x[half][j] * x[half][j];
      const float inv = rsqrtf(quad_sum(ss) / C + eps);
      if (!HEAD) {
        const int ch = 4 * c;
        if (F32) {
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(pixels) + px * C + ch) =
              make_float4(x[half][0], x[half][1], x[half][2], x[half][3]);
        } else {
          *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(pixels) + px * C + ch) =
              make_uint2(pack_bf16x2(x[half][0], x[half][1]), pack_bf16x2(x[half][2], x[half][3]));
        }
        *reinterpret_cast<uint2*>(next_input + px * C + ch) =
            make_uint2(pack_bf16x2(x[half][0] * inv * gain_next[0], x[half][1] * inv * gain_next[1]),
                       pack_bf16x2(x[half][2] * inv * gain_next[2], x[half][3] * inv * gain_next[3]));
      } else {
        float part[3] = {0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float hn = F32 ? x[half][j] * inv * gain_next[j] : round_bf16(x[half][j] * inv * gain_next[j]);
          const int ch = 4 * c + j;
#pragma unroll
          for (int o = 0; o < 3; ++o) part[o] = fmaf(hn, __ldg(fw + o * C + ch), part[o]);
        }
#pragma unroll
        for (int o = 0; o < 3; ++o) part[o] = quad_sum(part[o]);
        if (c == 0) {  // pixel k0 + g + 8 half of the tile's patch: row k / patch, column k % patch
          const int k = fold.k0 + g + 8 * half;
          const int ky = k / patch;
          float* dst = v + fold.base + static_cast<int64_t>(ky) * width + (k - ky * patch);
#pragma unroll
          for (int o = 0; o < 3; ++o) dst[o * fold.plane] = part[o] + __ldg(fb + o);
        }
      }
    }
  };

  // this warp's tiles: first, first + warps, ...; MMA_RING - 1 of them in flight ahead
  const int64_t first = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int64_t count = first < tiles ? (tiles - 1 - first) / warps + 1 : 0;
#pragma unroll
  for (int s = 0; s < MMA_RING - 1; ++s) {
    if (s < count) issue_tile(first + s * warps, s);
    cp_async_commit();  // one group per tile, empty past the last, so the wait counts stay fixed
  }
  for (int64_t i = 0; i < count; ++i) {
    __syncwarp();  // every lane is done reading the slot refilled next
    const int64_t ahead = i + MMA_RING - 1;
    if (ahead < count) issue_tile(first + ahead * warps, static_cast<int>(ahead % MMA_RING));
    cp_async_commit();
    cp_async_wait<MMA_RING - 1>();  // tile i's group has landed for this lane
    __syncwarp();                   // and for every lane
    TileIn in;
    read_tile(static_cast<int>(i % MMA_RING), in);
    process(first + i * warps, in);
  }
  cp_async_wait<0>();
}

__global__ void __launch_bounds__(THREADS) pixel_rms_norm_kernel(const void* pixels, bool f32,
                                                                  __nv_bfloat16* __restrict__ out,
                                                                  const float* __restrict__ weight, int64_t n,
                                                                  float eps) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float x[C];
    load16(pixels, i, f32, x);
    const float inv = inv_rms16(x, eps);
#pragma unroll
    for (int c = 0; c < C; ++c) x[c] = x[c] * inv * __ldg(weight + c);
    store16(out, i, false, x);
  }
}

template <bool F32>
__global__ void __launch_bounds__(THREADS) pixel_mlp_kernel(void* pixels, const __nv_bfloat16* __restrict__ branch,
                                                             const __nv_bfloat16* __restrict__ mods,
                                                             const float* nw, const __nv_bfloat16* w1,
                                                             const __nv_bfloat16* b1, const __nv_bfloat16* w2,
                                                             const __nv_bfloat16* b2, const float* nnw,
                                                             __nv_bfloat16* __restrict__ next_input, int64_t n,
                                                             float eps) {
  __shared__ MlpWeights s;
  load_weights(s, w1, b1, w2, b2, nw, nnw, nullptr, nullptr);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float x[C], attn[C];
    load16(pixels, i, F32, x);
    load16(branch, i, false, attn);
    pit_tail<!F32>(x, attn, mods + i * 4 * C, s, eps);
    store16(pixels, i, F32, x);
    const float inv = inv_rms16(x, eps);
    float y[C];
#pragma unroll
    for (int c = 0; c < C; ++c) y[c] = x[c] * inv * s.nnw[c];
    store16(next_input, i, false, y);
  }
}

template <bool F32>
__global__ void __launch_bounds__(THREADS) pixel_mlp_head_kernel(
    const void* pixels, const __nv_bfloat16* __restrict__ branch, const __nv_bfloat16* __restrict__ mods,
    const float* nw, const __nv_bfloat16* w1, const __nv_bfloat16* b1, const __nv_bfloat16* w2,
    const __nv_bfloat16* b2, const float* fnw, const float* fw, const float* fb, float* __restrict__ v, int64_t n,
    int64_t height, int64_t width, int patch, int64_t token_start, int64_t tokens, float eps) {
  __shared__ MlpWeights s;
  load_weights(s, w1, b1, w2, b2, nw, fnw, fw, fb);
  const int pp = patch * patch;
  const int64_t gw = width / patch;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float x[C], attn[C];
    load16(pixels, i, F32, x);
    load16(branch, i, false, attn);
    pit_tail<!F32>(x, attn, mods + i * 4 * C, s, eps);
    const float inv = inv_rms16(x, eps);
    float h[C];
#pragma unroll
    for (int c = 0; c < C; ++c) h[c] = F32 ? x[c] * inv * s.nnw[c] : round_bf16(x[c] * inv * s.nnw[c]);
    const int64_t patch_idx = i / pp;
    const int k = static_cast<int>(i % pp);
    const int64_t b = patch_idx / tokens, l = token_start + patch_idx % tokens;
    const int64_t y = (l / gw) * patch + k / patch, xx = (l % gw) * patch + k % patch;
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
      float acc = s.fb[ch];
#pragma unroll
      for (int c = 0; c < C; ++c) acc = fmaf(h[c], s.fw[ch * C + c], acc);
      v[((b * 3 + ch) * height + y) * width + xx] = acc;
    }
  }
}

__global__ void __launch_bounds__(THREADS) pixel_embed_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                               const float* __restrict__ bias,
                                                               const float* __restrict__ pos, void* pixels, bool f32,
                                                               __nv_bfloat16* __restrict__ normed,
                                                               const float* __restrict__ nw, float eps, int64_t n,
                                                               int channels, int64_t height, int64_t width,
                                                               int patch, int64_t token_start, int64_t tokens) {
  // W [16, channels] (nn.Linear layout), then the bias and the norm gain
  __shared__ float sw[MAX_IN_CHANNELS * C + C + C];
  float* sb = sw + MAX_IN_CHANNELS * C;
  float* sn = sb + C;
  for (int i = threadIdx.x; i < channels * C; i += blockDim.x) sw[i] = w[i];
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    sb[i] = bias[i];
    sn[i] = nw[i];
  }
  __syncthreads();
  const int pp = patch * patch;
  const int64_t gw = width / patch;
  const int64_t plane = height * width;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t patch_idx = i / pp;
    const int k = static_cast<int>(i % pp);
    const int64_t b = patch_idx / tokens, l = token_start + patch_idx % tokens;
    const int64_t y = (l / gw) * patch + k / patch, xx = (l % gw) * patch + k % patch;
    const float* xp = x + b * channels * plane + y * width + xx;
    float xin[MAX_IN_CHANNELS];
#pragma unroll
    for (int k = 0; k < MAX_IN_CHANNELS; ++k) xin[k] = k < channels ? xp[k * plane] : 0.f;
    float o[C];
#pragma unroll
    for (int c = 0; c < C; ++c) {
      // F.linear(x, W, b): sum over the input channels in order, then the bias
      const float* wc = sw + c * channels;
      float acc = xin[0] * wc[0];
#pragma unroll
      for (int k = 1; k < MAX_IN_CHANNELS; ++k)
        if (k < channels) acc = fmaf(xin[k], wc[k], acc);
      o[c] = acc + sb[c];
    }
    if (pos != nullptr) {
      const float4* p4 = reinterpret_cast<const float4*>(pos + (y * width + xx) * C);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 pv = __ldg(p4 + j);
        o[4 * j] += pv.x; o[4 * j + 1] += pv.y; o[4 * j + 2] += pv.z; o[4 * j + 3] += pv.w;
      }
    }
    if (!f32) {
#pragma unroll
      for (int c = 0; c < C; ++c) o[c] = round_bf16(o[c]);
    }
    store16(pixels, i, f32, o);
    const float inv = inv_rms16(o, eps);
    float h[C];
#pragma unroll
    for (int c = 0; c < C; ++c) h[c] = o[c] * inv * sn[c];
    store16(normed, i, false, h);
  }
}

inline unsigned grid_for(int64_t n) {
  int64_t blocks = (n + THREADS - 1) / THREADS;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
  return static_cast<unsigned>(blocks < cap ? blocks : cap);
}

// 16-pixel tiles, one per warp, 4 warps per block, grid-stride beyond the
// resident blocks (MMA_BLOCKS_PER_SM)
inline unsigned mma_grid_for(int64_t n) {
  const int64_t blocks = (n / 16 + MMA_THREADS / 32 - 1) / (MMA_THREADS / 32);
  const int64_t cap = static_cast<int64_t>(num_sms()) * MMA_BLOCKS_PER_SM;
  return static_cast<unsigned>(blocks < cap ? blocks : cap);
}

}  // namespace pixel
}  // namespace iris

using namespace iris;

static int check_pixel_params(const void* w1, const void* b1, const void* w2, const void* b2, const float* nw) {
  IRIS_REQUIRE(w1 && b1 && w2 && b2 && nw, "pixel_mlp_ needs the released pixel-stage widths");
  return IRIS_OK;
}

extern "C" int iris_pixel_rms_norm(const void* pixels, int pixel_dtype, void* out, const float* weight,
                                   int64_t n_pixels, float eps, void* stream) {
  using namespace iris::pixel;
  IRIS_REQUIRE(pixels && out && weight, "pixel_rms_norm gain width mismatch (null pointer)");
  IRIS_REQUIRE(pixel_dtype == IRIS_F32 || pixel_dtype == IRIS_BF16, "pixel_rms_norm: pixels must be f32 or bf16");
  IRIS_REQUIRE(aligned16(pixels) && aligned16(out), "pixel_rms_norm: pointers must be 16-byte aligned");
  IRIS_REQUIRE(n_pixels >= 0, "pixel_rms_norm: negative size");
  if (n_pixels == 0) return IRIS_OK;
  pixel_rms_norm_kernel<<<grid_for(n_pixels), THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      pixels, pixel_dtype == IRIS_F32, reinterpret_cast<__nv_bfloat16*>(out), weight, n_pixels, eps);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_pixel_mlp(void* pixels, int pixel_dtype, const void* branch, const void* mods,
                              const float* norm_weight, const void* fc1_w, const void* fc1_b, const void* fc2_w,
                              const void* fc2_b, const float* next_norm_weight, void* next_input, int64_t n_pixels,
                              float eps, void* stream) {
  using namespace iris::pixel;
  IRIS_REQUIRE(pixels && branch && mods && next_input && next_norm_weight, "pixel_mlp_: null pointer");
  IRIS_CHECK_STATUS(check_pixel_params(fc1_w, fc1_b, fc2_w, fc2_b, norm_weight));
  IRIS_REQUIRE(pixel_dtype == IRIS_F32 || pixel_dtype == IRIS_BF16, "pixel_mlp_: pixels must be f32 or bf16");
  IRIS_REQUIRE(aligned16(pixels) && aligned16(branch) && aligned16(mods) && aligned16(next_input),
               "pixel_mlp_: activations must be 16-byte aligned");
  IRIS_REQUIRE(n_pixels >= 0, "pixel_mlp_: negative size");
  if (n_pixels == 0) return IRIS_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto bf = [](const void* p) { return reinterpret_cast<const __nv_bfloat16*>(p); };
  if (n_pixels % 16 == 0) {  // whole 16-pixel tiles: tensor-core MLP
    const unsigned grid = mma_grid_for(n_pixels);
    auto nxt = reinterpret_cast<__nv_bfloat16*>(next_input);
    if (pixel_dtype == IRIS_F32) {
      IRIS_CUDA(cudaFuncSetAttribute(pixel_mlp_mma_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     mma_smem_bytes(true)));
      pixel_mlp_mma_kernel<true, false><<<grid, MMA_THREADS, mma_smem_bytes(true), st>>>(
          pixels, bf(branch), bf(mods), norm_weight, bf(fc1_w), bf(fc1_b), bf(fc2_w), bf(fc2_b), next_norm_weight,
          nxt, nullptr, nullptr, nullptr, n_pixels, 16, 16, 16, 0, 1, eps);
    } else {
      IRIS_CUDA(cudaFuncSetAttribute(pixel_mlp_mma_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     mma_smem_bytes(false)));
      pixel_mlp_mma_kernel<false, false><<<grid, MMA_THREADS, mma_smem_bytes(false), st>>>(
          pixels, bf(branch), bf(mods), norm_weight, bf(fc1_w), bf(fc1_b), bf(fc2_w), bf(fc2_b), next_norm_weight,
          nxt, nullptr, nullptr, nullptr, n_pixels, 16, 16, 16, 0, 1, eps);
    }
    IRIS_CUDA(cudaGetLastError());
    return IRIS_OK;
  }
  if (pixel_dtype == IRIS_F32)
    pixel_mlp_kernel<true><<<grid_for(n_pixels), THREADS, 0, st>>>(
        pixels, bf(branch), bf(mods), norm_weight, bf(fc1_w), bf(fc1_b), bf(fc2_w), bf(fc2_b), next_norm_weight,
        reinterpret_cast<__nv_bfloat16*>(next_input), n_pixels, eps);
  else
    pixel_mlp_kernel<false><<<grid_for(n_pixels), THREADS, 0, st>>>(
        pixels, bf(branch), bf(mods), norm_weight, bf(fc1_w), bf(fc1_b), bf(fc2_w), bf(fc2_b), next_norm_weight,
        reinterpret_cast<__nv_bfloat16*>(next_input), n_pixels, eps);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_pixel_mlp_head(void* pixels, int pixel_dtype, const void* branch, const void* mods,
                                   const float* norm_weight, const void* fc1_w, const void* fc1_b, const void* fc2_w,
                                   const void* fc2_b, const float* final_norm_weight, const float* final_w,
                                   const float* final_b, float* v, int64_t batch, int64_t height, int64_t width,
                                   int64_t patch, int64_t token_start, int64_t tokens, float eps, void* stream) {
  using namespace iris::pixel;
  IRIS_REQUIRE(pixels && branch && mods && final_norm_weight && final_w && final_b && v, "pixel_mlp_head: null pointer");
  IRIS_CHECK_STATUS(check_pixel_params(fc1_w, fc1_b, fc2_w, fc2_b, norm_weight));
  IRIS_REQUIRE(pixel_dtype == IRIS_F32 || pixel_dtype == IRIS_BF16, "pixel_mlp_head: pixels must be f32 or bf16");
  IRIS_REQUIRE(patch > 0 && height % patch == 0 && width % patch == 0 && batch >= 0, "pixel_mlp_head: bad geometry");
  IRIS_REQUIRE(aligned16(pixels) && aligned16(branch) && aligned16(mods), "pixel_mlp_head: alignment");
  IRIS_REQUIRE(token_start >= 0 && tokens >= 0 && token_start + tokens <= (height / patch) * (width / patch),
               "pixel_mlp_head: token range outside the patch grid");
  const int64_t n = batch * tokens * patch * patch;
  if (n == 0) return IRIS_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto bf = [](const void* p) { return reinterpret_cast<const __nv_bfloat16*>(p); };
  if (n % 16 == 0 && patch % 4 == 0) {  // whole 16-pixel tiles, each inside one patch: tensor-core MLP
    const unsigned grid = mma_grid_for(n);
    const int pt = static_cast<int>(patch);
    if (pixel_dtype == IRIS_F32) {
      IRIS_CUDA(cudaFuncSetAttribute(pixel_mlp_mma_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     mma_smem_bytes(true)));
      pixel_mlp_mma_kernel<true, true><<<grid, MMA_THREADS, mma_smem_bytes(true), st>>>(
          pixels, bf(branch), bf(mods), norm_weight, bf(fc1_w), bf(fc1_b), bf(fc2_w), bf(fc2_b), final_norm_weight,
          nullptr, final_w, final_b, v, n, height, width, pt, token_start, tokens, eps);
    } else {
      IRIS_CUDA(cudaFuncSetAttribute(pixel_mlp_mma_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     mma_smem_bytes(false)));
      pixel_mlp_mma_kernel<false, true><<<grid, MMA_THREADS, mma_smem_bytes(false), st>>>(
          pixels, bf(branch), bf(mods), norm_weight, bf(fc1_w), bf(fc1_b), bf(fc2_w), bf(fc2_b), final_norm_weight,
          nullptr, final_w, final_b, v, n, height, width, pt, token_start, tokens, eps);
    }
    IRIS_CUDA(cudaGetLastError());
    return IRIS_OK;
  }
  if (pixel_dtype == IRIS_F32)
    pixel_mlp_head_kernel<true><<<grid_for(n), THREADS, 0, st>>>(
        pixels, bf(branch), bf(mods), norm_weight, bf(fc1_w), bf(fc1_b), bf(fc2_w), bf(fc2_b), final_norm_weight,
        final_w, final_b, v, n, height, width, static_cast<int>(patch), token_start, tokens, eps);
  else
    pixel_mlp_head_kernel<false><<<grid_for(n), THREADS, 0, st>>>(
        pixels, bf(branch), bf(mods), norm_weight, bf(fc1_w), bf(fc1_b), bf(fc2_w), bf(fc2_b), final_norm_weight,
        final_w, final_b, v, n, height, width, static_cast<int>(patch), token_start, tokens, eps);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_pixel_embed(const float* x, const float* w, const float* bias, const float* pos, void* pixels,
                                int pixel_dtype, void* normed, const float* norm_weight, float eps, int64_t batch,
                                int64_t channels, int64_t height, int64_t width, int64_t patch, int64_t token_start,
                                int64_t tokens, void* stream) {
  using namespace iris::pixel;
  IRIS_REQUIRE(x && w && bias && pixels && normed && norm_weight, "pixel_embed: null pointer");
  IRIS_REQUIRE(channels >= 1 && channels <= MAX_IN_CHANNELS, "pixel_embed: 1 to 4 input channels");
  IRIS_REQUIRE(pixel_dtype == IRIS_F32 || pixel_dtype == IRIS_BF16, "pixel_embed: pixels must be f32 or bf16");
  IRIS_REQUIRE(patch > 0 && height % patch == 0 && width % patch == 0 && batch >= 0, "pixel_embed: bad geometry");
  IRIS_REQUIRE(aligned16(pixels) && aligned16(normed) && (pos == nullptr || aligned16(pos)), "pixel_embed: alignment");
  IRIS_REQUIRE(token_start >= 0 && tokens >= 0 && token_start + tokens <= (height / patch) * (width / patch),
               "pixel_embed: token range outside the patch grid");
  const int64_t n = batch * tokens * patch * patch;
  if (n == 0) return IRIS_OK;
  pixel_embed_kernel<<<grid_for(n), THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      x, w, bias, pos, pixels, pixel_dtype == IRIS_F32, reinterpret_cast<__nv_bfloat16*>(normed), norm_weight, eps, n,
      static_cast<int>(channels), height, width, static_cast<int>(patch), token_start, tokens);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}
