// Flash attention forward on the 5th-generation tensor cores: non-causal,
// unmasked softmax(Q K^T / sqrt(128)) V over the joint [text | image] sequence
// (src/iris_metal/model.py:243-250; src/iris3b/nn/attention.py:61-91) and the
// pixel-stage patch tokens (src/iris3b/models/blocks/pit.py:66-72).
//
// One CTA per (128-query tile, head, batch). Warp roles:
//   warp 0      TMA: Q once (two 64-dim halves, 128B swizzle), then K_j and V_j
//               (128 keys each) into 2-stage rings;
//   warp 1      TMEM allocator + MMA issuer (one thread):
//                 S[j % 2]  = Q K_j^T          (SS MMA, M=N=128, K=128)
//                 O        += P[j % 2] V_j     (TS MMA, P read from TMEM)
//               S_{j+1} is issued before O += P_j V_j so the tensor pipe
//               works on the next scores while the softmax warps run;
//   warps 2..5  softmax, one query row per thread (TMEM lane = row): load the
//               row of S, running max / sum in fp32 (exp2 domain), write P as
//               packed bf16 into TMEM; rescale O in TMEM only when the row max
//               grew by more than 2^8 (the stale max is exact at the end since
//               O and l share it); final O / l -> bf16 -> [b, n, h*128 + d].
// TMEM: S0 [0,128) S1 [128,256) O [256,384) P0 [384,448) P1 [448,512).
#include "common.cuh"
#include "iris_abi_internal.h"

namespace iris {
namespace attn {

constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int D = 128;
constexpr int HALF_BYTES = 128 * 64 * 2;  // 128 rows x 64 dims, 16 KB
constexpr int TILE_BYTES = 2 * HALF_BYTES;  // 32 KB
constexpr int THREADS = 192;
constexpr uint32_t COL_S = 0, COL_O = 256, COL_P = 384;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units
constexpr size_t SMEM_BYTES = 1024 + 5 * TILE_BYTES + 256;

struct Smem {
  uint64_t q_full;
  uint64_t k_full[2], k_free[2], v_full[2], v_free[2];
  uint64_t s_full[2], s_free[2], p_full[2];
  uint64_t o_done;
  uint64_t teardown;
  uint32_t tmem_base;
  int abort;
};

struct Params {
  int64_t batch, heads_q, heads_kv, n, o_row_stride;
  float scale_log2;
  __nv_bfloat16* o;
};

IRIS_DEVICE float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(THREADS, 1)
    flash_attn_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                      const __grid_constant__ CUtensorMap tv, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_tile = base;
  uint8_t* k_tile = base + TILE_BYTES;      // 2 stages
  uint8_t* v_tile = base + 3 * TILE_BYTES;  // 2 stages
  Smem* s = reinterpret_cast<Smem*>(base + 5 * TILE_BYTES);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int q_tile_idx = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int group = static_cast<int>(p.heads_q / p.heads_kv);
  const int hk = h / group;
  const int n = static_cast<int>(p.n);
  const int nkv = (n + BKV - 1) / BKV;
  const int q_row0 = static_cast<int>((static_cast<int64_t>(b) * p.heads_q + h) * n) + q_tile_idx * BQ;
  const int kv_row0 = static_cast<int>((static_cast<int64_t>(b) * p.heads_kv + hk) * n);

  if (threadIdx.x == 0) {
    mbar_init(&s->q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s->k_full[i], 1);
      mbar_init(&s->k_free[i], 1);
      mbar_init(&s->v_full[i], 1);
      mbar_init(&s->v_free[i], 1);
      mbar_init(&s->s_full[i], 1);
      mbar_init(&s->s_free[i], 4);
      mbar_init(&s->p_full[i], 4);
    }
    mbar_init(&s->o_done, 1);
    mbar_init(&s->teardown, 1);
    s->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&s->tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s->tmem_base;
  volatile int* abort = &s->abort;

  if (warp == 0) {
    // ----------------------------------------------------------------- TMA
    if (lane == 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      mbar_arrive_expect_tx(&s->q_full, TILE_BYTES);
      tma_load_2d(&tq, &s->q_full, q_tile, 0, q_row0);
      tma_load_2d(&tq, &s->q_full, q_tile + HALF_BYTES, 64, q_row0);
      int issued_k[2] = {-1, -1}, issued_v[2] = {-1, -1};
      bool ok = true;
      for (int j = 0; j < nkv && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = static_cast<uint32_t>((j >> 1) & 1);
        const int row = kv_row0 + j * BKV;
        if (!mbar_wait(&s->k_free[st], ph ^ 1u, abort)) { ok = false; break; }
        mbar_arrive_expect_tx(&s->k_full[st], TILE_BYTES);
        tma_load_2d(&tk, &s->k_full[st], k_tile + st * TILE_BYTES, 0, row);
        tma_load_2d(&tk, &s->k_full[st], k_tile + st * TILE_BYTES + HALF_BYTES, 64, row);
        issued_k[st] = static_cast<int>(ph);
        if (!mbar_wait(&s->v_free[st], ph ^ 1u, abort)) { ok = false; break; }
        mbar_arrive_expect_tx(&s->v_full[st], TILE_BYTES);
        tma_load_2d(&tv, &s->v_full[st], v_tile + st * TILE_BYTES, 0, row);
        tma_load_2d(&tv, &s->v_full[st], v_tile + st * TILE_BYTES + HALF_BYTES, 64, row);
        issued_v[st] = static_cast<int>(ph);
      }
      if (!ok) {
        int dummy = 0;
        mbar_wait(&s->q_full, 0, &dummy);
        for (int i = 0; i < 2; ++i) {
          if (issued_k[i] >= 0) mbar_wait(&s->k_full[i], static_cast<uint32_t>(issued_k[i]), &dummy);
          if (issued_v[i] >= 0) mbar_wait(&s->v_full[i], static_cast<uint32_t>(issued_v[i]), &dummy);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t idesc_s = idesc_bf16_f32(BQ, BKV);
      const uint32_t idesc_o = idesc_bf16_f32(BQ, D, false, true);  // V is MN-major (dims contiguous)
      const uint32_t q_addr = smem_addr(q_tile);
      bool ok = mbar_wait(&s->q_full, 0, abort);
      // S_j = Q K_j^T into S[j % 2]
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        const uint32_t ph = static_cast<uint32_t>((j >> 1) & 1);
        if (!mbar_wait(&s->k_full[st], ph, abort)) return false;
        if (!mbar_wait(&s->s_free[st], ph ^ 1u, abort)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_addr(k_tile + st * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
          const uint64_t ad = umma_desc(q_addr + off, 16, 1024, kLayoutSw128);
          const uint64_t bd = umma_desc(k_addr + off, 16, 1024, kLayoutSw128);
          umma_ss(tmem + COL_S + st * BKV, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s->s_full[st]);
        umma_commit(&s->k_free[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < nkv && ok; ++j) {
        if (j + 1 < nkv && !issue_s(j + 1)) { ok = false; break; }
        const int st = j & 1;
        const uint32_t ph = static_cast<uint32_t>((j >> 1) & 1);
        if (!mbar_wait(&s->p_full[st], ph, abort) || !mbar_wait(&s->v_full[st], ph, abort)) { ok = false; break; }
        tc_fence_after();
        const uint32_t v_addr = smem_addr(v_tile + st * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          // 16 keys per MMA: 16 rows of 128 B in the swizzled V tile, 8 packed P columns
          const uint64_t bd = umma_desc(v_addr + kk * 16 * 128, HALF_BYTES, 1024, kLayoutSw128);
          umma_ts(tmem + COL_O, tmem + COL_P + st * 64 + kk * 8, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&s->o_done);
        umma_commit(&s->v_free[st]);
      }
      umma_commit(&s->teardown);
      int dummy = 0;
      mbar_wait(&s->teardown, 0, &dummy);
    }
  } else {
    // ------------------------------------------------------------- softmax
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int st = j & 1;
      const uint32_t ph = static_cast<uint32_t>((j >> 1) & 1);
      if (!__all_sync(0xffffffffu, mbar_wait(&s->s_full[st], ph, abort))) { ok = false; break; }
      tc_fence_after();
      float sv[BKV];
      {
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          tmem_ld32(tmem + lane_addr + COL_S + st * BKV + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) sv[c * 32 + e] = __uint_as_float(r[e]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s->s_free[st]);
      // scores in log2 units, keys past the sequence end masked out
      const int valid = n - j * BKV;
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < BKV; ++e) {
        sv[e] = e < valid ? sv[e] * p.scale_log2 : -INFINITY;
        mx = fmaxf(mx, sv[e]);
      }
      const bool grow = mx > m_run + RESCALE_THRESHOLD;
      const bool rescale = __any_sync(0xffffffffu, grow) && j > 0;
      float m_new = m_run;
      if (grow || j == 0) m_new = fmaxf(m_run, mx);
      if (rescale && !grow) m_new = m_run;  // this row keeps its max; the warp rescales O together
      const float corr = (j == 0) ? 0.f : ex2(m_run - m_new);
      float rs = 0.f;
      // PV_{j-1} must be done before O is rescaled or P[st] (read by PV_{j-2}) is overwritten
      if (j > 0) {
        if (!__all_sync(0xffffffffu, mbar_wait(&s->o_done, static_cast<uint32_t>((j - 1) & 1), abort))) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float p0 = ex2(sv[c * 32 + 2 * e] - m_new);
          const float p1 = ex2(sv[c * 32 + 2 * e + 1] - m_new);
          rs += p0 + p1;
          pk[e] = pack_bf16x2(p0, p1);
        }
        tmem_st16(tmem + lane_addr + COL_P + st * 64 + c * 16, pk);
      }
      l_run = (j == 0) ? rs : l_run * corr + rs;
      if (rescale) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_addr + COL_O + c * 32, r);
          tmem_wait_ld();
          uint32_t lo[16], hi[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            lo[e] = __float_as_uint(__uint_as_float(r[e]) * corr);
            hi[e] = __float_as_uint(__uint_as_float(r[16 + e]) * corr);
          }
          tmem_st16(tmem + lane_addr + COL_O + c * 32, lo);
          tmem_st16(tmem + lane_addr + COL_O + c * 32 + 16, hi);
        }
      }
      m_run = m_new;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s->p_full[st]);
    }
    if (ok && __all_sync(0xffffffffu, mbar_wait(&s->o_done, static_cast<uint32_t>((nkv - 1) & 1), abort))) {
      tc_fence_after();
      const int q = q_tile_idx * BQ + row;
      const float inv = 1.f / l_run;
      __nv_bfloat16* dst = p.o + (static_cast<int64_t>(b) * p.n + q) * p.o_row_stride + static_cast<int64_t>(h) * D;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_addr + COL_O + c * 32, r);
        tmem_wait_ld();
        if (q < n) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            d4[e] = make_uint4(pack_bf16x2(__uint_as_float(r[8 * e]) * inv, __uint_as_float(r[8 * e + 1]) * inv),
                               pack_bf16x2(__uint_as_float(r[8 * e + 2]) * inv, __uint_as_float(r[8 * e + 3]) * inv),
                               pack_bf16x2(__uint_as_float(r[8 * e + 4]) * inv, __uint_as_float(r[8 * e + 5]) * inv),
                               pack_bf16x2(__uint_as_float(r[8 * e + 6]) * inv, __uint_as_float(r[8 * e + 7]) * inv));
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

}  // namespace attn
}  // namespace iris

using namespace iris;

extern "C" int iris_flash_attn_fwd(const void* q, const void* k, const void* v, void* o, int64_t batch,
                                   int64_t heads_q, int64_t heads_kv, int64_t n, int64_t head_dim, float scale,
                                   int64_t o_row_stride, void* stream) {
  using namespace iris::attn;
  IRIS_REQUIRE(q && k && v && o, "flash_attn_fwd: null pointer");
  IRIS_REQUIRE(head_dim == D, "flash_attn_fwd: head_dim must be 128");
  IRIS_REQUIRE(batch > 0 && heads_q > 0 && heads_kv > 0 && heads_q % heads_kv == 0,
               "flash_attn_fwd: heads_q must be a positive multiple of heads_kv");
  IRIS_REQUIRE(n > 0 && batch * heads_q * n < (1ll << 31), "flash_attn_fwd: sequence too long");
  IRIS_REQUIRE(o_row_stride >= heads_q * D && o_row_stride % 8 == 0, "flash_attn_fwd: o_row_stride");
  IRIS_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o), "flash_attn_fwd: alignment");
  IRIS_REQUIRE(batch <= 65535 && heads_q <= 65535, "flash_attn_fwd: grid too large");
  CUtensorMap tq, tk, tv;
  IRIS_CHECK_STATUS(make_tmap_2d_bf16(&tq, q, D, batch * heads_q * n, D, 64, BQ));
  IRIS_CHECK_STATUS(make_tmap_2d_bf16(&tk, k, D, batch * heads_kv * n, D, 64, BKV));
  IRIS_CHECK_STATUS(make_tmap_2d_bf16(&tv, v, D, batch * heads_kv * n, D, 64, BKV));
  Params p;
  p.batch = batch;
  p.heads_q = heads_q;
  p.heads_kv = heads_kv;
  p.n = n;
  p.o_row_stride = o_row_stride;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  static bool configured[64] = {false};
  int dev = 0;
  IRIS_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && !configured[dev]) {
    IRIS_CUDA(cudaFuncSetAttribute(flash_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(SMEM_BYTES)));
    configured[dev] = true;
  }
  dim3 grid(static_cast<unsigned>((n + BQ - 1) / BQ), static_cast<unsigned>(heads_q), static_cast<unsigned>(batch));
  flash_attn_kernel<<<grid, THREADS, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}
