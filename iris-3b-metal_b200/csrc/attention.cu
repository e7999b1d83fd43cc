// Flash attention forward on the 5th-generation tensor cores: non-causal,
// unmasked softmax(Q K^T / sqrt(128)) V over the joint [text | image] sequence
// (src/iris_metal/model.py:243-250; src/iris3b/nn/attention.py:61-91) and the
// pixel-stage patch tokens (src/iris3b/models/blocks/pit.py:66-72). Queries
// and keys may differ in number (a sequence-parallel rank attends with its own
// patch tokens over the gathered keys of all of them).
//
// One CTA per (256 queries = two 128-row tiles, head, batch). Warp roles:
//   warp 0      TMA: both Q tiles once (two 64-dim halves each, 128B swizzle),
//               then K_j and V_j (128 keys each) into 2-stage rings;
//   warp 1      TMEM allocator + MMA issuer (one thread). Per key block j the
//               tensor pipe runs, in order,
//                 O_0 += P_0 V_j,  S_0 = Q_0 K_{j+1}^T,  O_1 += P_1 V_j,  S_1 = Q_1 K_{j+1}^T
//               so one tile's softmax overlaps the other tile's MMAs;
//   warps 2..9  softmax of tile 0, warps 10..17 softmax of tile 1. A query row
//               (TMEM lane) is shared by two warps, one per half of the 128 key
//               columns; they combine the row max and sum through shared memory
//               (a 64-thread named barrier per lane quarter). Running max / sum
//               in fp32 in the exp2 domain; each half writes its P as packed
//               bf16 over the first 32 of its own 64 score columns in TMEM (read
//               by the next TS MMA, which completes before the following S MMA
//               overwrites them: the MMAs of one thread execute in issue order);
//               O is rescaled in TMEM only when a row max grew by more than 2^8
//               (O and l share the stale max, so the result is exact). With a
//               score bound (QK-normed heads), a row whose running max is within
//               2^64 of the bound keeps it: no later score can overflow P, and
//               the row-max pass and its exchange stop for the rest of the keys.
//               Final O / l (times the sigmoid gate, if any) -> bf16 rows per stream.
// TMEM: S_0 [0,128) S_1 [128,256) O_0 [256,384) O_1 [384,512).
#include "common.cuh"
#include "iris_abi_internal.h"

namespace iris {
namespace attn {

constexpr int BQ = 128;       // rows per query tile
constexpr int TILES = 2;      // query tiles per CTA
constexpr int BKV = 128;
constexpr int D = 128;
constexpr int HALF_BYTES = 128 * 64 * 2;  // 128 rows x 64 dims, 16 KB
constexpr int TILE_BYTES = 2 * HALF_BYTES;  // 32 KB
constexpr int SOFTMAX_WARPS_PER_TILE = 8;  // two warps per TMEM lane quarter, one per key-column half
constexpr int THREADS = 64 + TILES * SOFTMAX_WARPS_PER_TILE * 32;  // 576
constexpr uint32_t COL_S = 0, COL_O = 256;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units
// A row whose running max is within this many log2 units of the score bound
// keeps it for good: P <= 2^64, row sums <= 2^64 n_kv, all finite in fp32 / bf16.
constexpr float BOUND_MARGIN = 64.0f;
constexpr size_t SMEM_BYTES = 1024 + (TILES + 4) * TILE_BYTES + 8192;

struct Smem {
  uint64_t q_full;
  uint64_t k_full[2], k_free[2], v_full[2], v_free[2];
  uint64_t s_full[TILES], p_full[TILES], o_final[TILES];
  uint64_t teardown;
  uint32_t tmem_base;
  int abort;
  float row_max[2][TILES][2][BQ];  // [iteration parity][tile][column half][row]
  float row_sum[TILES][2][BQ];
};

struct Params {
  int64_t batch, heads_q, heads_kv, n, n_kv, row_stride, split;  // n queries and n_kv keys per (b, h)
  float scale_log2;
  // > 0: every score * scale_log2 is at most this (QK-normed heads bound it;
  // see iris_flash_attn_fwd_split); 0: no bound known
  float bound_log2;
  __nv_bfloat16* o_text;   // rows b * split + i       (i < split)
  __nv_bfloat16* o_image;  // rows b * (n - split) + i - split
  const __nv_bfloat16* gate_text;  // bf16 gate logits in the same rows, or null
  const __nv_bfloat16* gate_image;
  // sequence parallelism (peers > 0): query i's row goes to rank i / peer_tokens,
  // row b * peer_tokens + i % peer_tokens, columns peer_col0 + h * 128 ...
  int64_t peers, peer_tokens, peer_col0, peer_row_stride;
  __nv_bfloat16* o_peer[IRIS_MAX_PEERS];
};

IRIS_DEVICE float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed FP32 pair arithmetic (sm_100 f32x2 instructions): one issue, two lanes
// of work. The intrinsics keep the pair in a register pair, without moves.
IRIS_DEVICE float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
IRIS_DEVICE float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }

IRIS_DEVICE void named_barrier_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

IRIS_DEVICE float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__global__ void __launch_bounds__(THREADS, 1)
    flash_attn_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                      const __grid_constant__ CUtensorMap tv, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_tile = base;                             // TILES x 32 KB
  uint8_t* k_tile = base + TILES * TILE_BYTES;        // 2 stages
  uint8_t* v_tile = base + (TILES + 2) * TILE_BYTES;  // 2 stages
  Smem* s = reinterpret_cast<Smem*>(base + (TILES + 4) * TILE_BYTES);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int group = static_cast<int>(p.heads_q / p.heads_kv);
  const int hk = h / group;
  const int n = static_cast<int>(p.n);
  const int n_kv = static_cast<int>(p.n_kv);
  const int nkv = (n_kv + BKV - 1) / BKV;
  const int q0 = blockIdx.x * (TILES * BQ);  // first query of the CTA
  const int q_row0 = static_cast<int>((static_cast<int64_t>(b) * p.heads_q + h) * n) + q0;
  const int kv_row0 = static_cast<int>((static_cast<int64_t>(b) * p.heads_kv + hk) * n_kv);

  if (threadIdx.x == 0) {
    mbar_init(&s->q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s->k_full[i], 1);
      mbar_init(&s->k_free[i], 1);
      mbar_init(&s->v_full[i], 1);
      mbar_init(&s->v_free[i], 1);
    }
    for (int t = 0; t < TILES; ++t) {
      mbar_init(&s->s_full[t], 1);
      mbar_init(&s->p_full[t], SOFTMAX_WARPS_PER_TILE);
      mbar_init(&s->o_final[t], 1);
    }
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
      mbar_arrive_expect_tx(&s->q_full, TILES * TILE_BYTES);
      for (int t = 0; t < TILES; ++t) {
        tma_load_2d(&tq, &s->q_full, q_tile + t * TILE_BYTES, 0, q_row0 + t * BQ);
        tma_load_2d(&tq, &s->q_full, q_tile + t * TILE_BYTES + HALF_BYTES, 64, q_row0 + t * BQ);
      }
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
      // S_t = Q_t K_j^T into S_t
      auto issue_s = [&](int t, int j) {
        const uint32_t q_addr = smem_addr(q_tile + t * TILE_BYTES);
        const uint32_t k_addr = smem_addr(k_tile + (j & 1) * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * HALF_BYTES + (kk & 3) * 32;
          const uint64_t ad = umma_desc(q_addr + off, 16, 1024, kLayoutSw128);
          const uint64_t bd = umma_desc(k_addr + off, 16, 1024, kLayoutSw128);
          umma_ss(tmem + COL_S + t * BKV, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s->s_full[t]);
      };
      // O_t += P_t V_j. P of keys [0, 64) is packed bf16 in S_t columns [0, 32),
      // keys [64, 128) in columns [64, 96): each softmax half overwrites its own scores
      auto issue_pv = [&](int t, int j) {
        const uint32_t v_addr = smem_addr(v_tile + (j & 1) * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          const uint64_t bd = umma_desc(v_addr + kk * 16 * 128, HALF_BYTES, 1024, kLayoutSw128);
          const uint32_t p_col = COL_S + t * BKV + (kk >> 2) * 64 + (kk & 3) * 8;
          umma_ts(tmem + COL_O + t * D, tmem + p_col, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(&s->q_full, 0, abort) && mbar_wait(&s->k_full[0], 0, abort);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < TILES; ++t) issue_s(t, 0);
        umma_commit(&s->k_free[0]);
      }
      for (int j = 0; j < nkv && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = static_cast<uint32_t>((j >> 1) & 1);
        const bool more = j + 1 < nkv;
        if (!mbar_wait(&s->v_full[st], ph, abort)) { ok = false; break; }
        if (more && !mbar_wait(&s->k_full[(j + 1) & 1], static_cast<uint32_t>(((j + 1) >> 1) & 1), abort)) {
          ok = false;
          break;
        }
        for (int t = 0; t < TILES; ++t) {
          if (!mbar_wait(&s->p_full[t], static_cast<uint32_t>(j & 1), abort)) { ok = false; break; }
          tc_fence_after();
          issue_pv(t, j);
          if (!more) umma_commit(&s->o_final[t]);
          if (more) issue_s(t, j + 1);
        }
        if (!ok) break;
        umma_commit(&s->v_free[st]);
        if (more) umma_commit(&s->k_free[(j + 1) & 1]);
      }
      umma_commit(&s->teardown);
      int dummy = 0;
      mbar_wait(&s->teardown, 0, &dummy);
    }
  } else {
    // ------------------------------------------------------------- softmax
    // Warp w >= 2: tile (w - 2) / 8, column half ((w - 2) / 4) % 2, TMEM lane
    // quarter w % 4 (its rows). The two warps of a (tile, quarter) hold the
    // same 32 query rows, key columns [0, 64) and [64, 128) respectively, and
    // combine row maxima and sums through shared memory.
    const int sw = warp - 2;
    const int tile = sw / SOFTMAX_WARPS_PER_TILE;
    const int half = (sw / 4) & 1;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t bar_id = 1 + tile * 4 + quarter;  // named barrier of the two warps
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_col = COL_S + tile * BKV + half * 64;  // this half's 64 score columns
    const uint32_t o_col = COL_O + tile * D + half * 64;    // and 64 output columns
    float m_run = -INFINITY, l_run = 0.f;
    // Once the score bound is within BOUND_MARGIN of every running max of this
    // warp's rows, m_run is final and the row-max pass (with its exchange
    // between the two halves) is skipped. Both warps of a row pair hold the
    // same 32 running maxima, so they take the same branch at every block.
    bool settled = false;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(&s->s_full[tile], static_cast<uint32_t>(j & 1), abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int valid = n_kv - j * BKV - half * 64;  // keys of this half that exist
      const bool tail = valid < 64;
      float m_new = m_run, corr = 1.f;
      if (!settled) {
      // pass 1: this half's row max, combined with the other half's
      float mx;
      {
        uint32_t r[2][32];
        tmem_ld32(tmem + lane_addr + s_col, r[0]);
        tmem_ld32(tmem + lane_addr + s_col + 32, r[1]);
        tmem_wait_ld();
        float ma = -INFINITY, mb = -INFINITY, mc = -INFINITY, md = -INFINITY;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          if (tail) {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (c * 32 + e >= valid) r[c][e] = __float_as_uint(-INFINITY);
          }
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            ma = max3(ma, __uint_as_float(r[c][e]), __uint_as_float(r[c][e + 1]));
            mb = max3(mb, __uint_as_float(r[c][e + 2]), __uint_as_float(r[c][e + 3]));
            mc = max3(mc, __uint_as_float(r[c][e + 4]), __uint_as_float(r[c][e + 5]));
            md = max3(md, __uint_as_float(r[c][e + 6]), __uint_as_float(r[c][e + 7]));
          }
        }
        const float part = fmaxf(max3(ma, mb, mc), md);
        float* xchg = s->row_max[j & 1][tile][half];
        xchg[row] = part;
        named_barrier_sync(bar_id, 64);
        mx = fmaxf(part, s->row_max[j & 1][tile][half ^ 1][row]) * p.scale_log2;
      }
      // lazy rescale: keep the stale max unless it grew by more than 2^8
      const bool grow = j == 0 || mx > m_run + RESCALE_THRESHOLD;
      m_new = grow ? fmaxf(m_run, mx) : m_run;
      corr = ex2(m_run - m_new);  // 0 on the first block
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        // O_t holds the P V of earlier blocks: S_t(j) completing implies they completed
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_addr + o_col + c * 32, r);
          tmem_wait_ld();
          uint32_t lo[16], hi[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            lo[e] = __float_as_uint(__uint_as_float(r[e]) * corr);
            hi[e] = __float_as_uint(__uint_as_float(r[16 + e]) * corr);
          }
          tmem_st16(tmem + lane_addr + o_col + c * 32, lo);
          tmem_st16(tmem + lane_addr + o_col + c * 32 + 16, hi);
        }
      }
      }  // !settled
      // pass 2: P = 2^(s * scale - m) for this half; packed bf16 over its first 32 columns
      const float2 scale2 = make_float2(p.scale_log2, p.scale_log2);
      const float2 shift2 = make_float2(-m_new, -m_new);
      float2 rs2 = make_float2(0.f, 0.f);
      uint32_t buf[2][32];
      tmem_ld32(tmem + lane_addr + s_col, buf[0]);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_wait_ld();
        if (c == 0) tmem_ld32(tmem + lane_addr + s_col + 32, buf[1]);
        uint32_t(&r)[32] = buf[c];
        if (tail) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (c * 32 + e >= valid) r[e] = __float_as_uint(-INFINITY);
        }
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float2 sv = make_float2(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]));
          const float2 x = fma2(sv, scale2, shift2);
          // masked keys (-inf) give exact zeros
          const float2 pe = make_float2(ex2(x.x), ex2(x.y));
          rs2 = add2(rs2, pe);
          pk[e] = pack_bf16x2(pe.x, pe.y);
        }
        // chunk c's P goes to columns [16c, 16c + 16) of this half, scores already read
        tmem_st16(tmem + lane_addr + s_col + c * 16, pk);
      }
      l_run = l_run * corr + (rs2.x + rs2.y);
      m_run = m_new;
      if (!settled && p.bound_log2 > 0.f) settled = __all_sync(0xffffffffu, p.bound_log2 - m_run <= BOUND_MARGIN);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s->p_full[tile]);
    }
    // the row sum over both halves
    s->row_sum[tile][half][row] = l_run;
    named_barrier_sync(bar_id, 64);
    const float l_total = l_run + s->row_sum[tile][half ^ 1][row];
    // output row of this query and its gate logits, fetched while the last P V runs
    const int q = q0 + tile * BQ + row;
    const bool text = q < p.split;
    const int64_t orow = text ? static_cast<int64_t>(b) * p.split + q
                              : static_cast<int64_t>(b) * (p.n - p.split) + (q - p.split);
    const int64_t off = orow * p.row_stride + static_cast<int64_t>(h) * D + half * 64;
    const __nv_bfloat16* gate = text ? p.gate_text : p.gate_image;
    uint4 gate_row[8];
    if (gate != nullptr && q < n) {
      const uint4* g4 = reinterpret_cast<const uint4*>(gate + off);
#pragma unroll
      for (int e = 0; e < 8; ++e) gate_row[e] = g4[e];
    }
    if (ok && __all_sync(0xffffffffu, mbar_wait(&s->o_final[tile], 0, abort))) {
      tc_fence_after();
      __nv_bfloat16* dst = (text ? p.o_text : p.o_image) + off;
      if (p.peers > 0) {  // the row of the rank that owns token q, over NVLink
        const int64_t owner = min(static_cast<int64_t>(q) / p.peer_tokens, p.peers - 1);
        const int64_t lrow = static_cast<int64_t>(b) * p.peer_tokens + (q - owner * p.peer_tokens);
        dst = p.o_peer[owner] + lrow * p.peer_row_stride + p.peer_col0 + static_cast<int64_t>(h) * D + half * 64;
      }
      const float inv = 1.f / l_total;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_addr + o_col + c * 32, r);
        tmem_wait_ld();
        if (q < n) {
          float val[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) val[e] = __uint_as_float(r[e]) * inv;
          if (gate != nullptr) {  // out = attn * sigmoid(gate logit), src/iris_metal/model.py:282-283
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint4 gv = gate_row[c * 4 + e];
              const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
              for (int hh = 0; hh < 4; ++hh) {
                const float2 lg = unpack_bf16x2(gw[hh]);
                val[8 * e + 2 * hh] *= 1.f / (1.f + __expf(-lg.x));
                val[8 * e + 2 * hh + 1] *= 1.f / (1.f + __expf(-lg.y));
              }
            }
          }
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            d4[e] = make_uint4(pack_bf16x2(val[8 * e], val[8 * e + 1]), pack_bf16x2(val[8 * e + 2], val[8 * e + 3]),
                               pack_bf16x2(val[8 * e + 4], val[8 * e + 5]), pack_bf16x2(val[8 * e + 6], val[8 * e + 7]));
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

static int launch_attention(const void* q, const void* k, const void* v, iris::attn::Params& p, void* stream) {
  using namespace iris::attn;
  CUtensorMap tq, tk, tv;
  IRIS_CHECK_STATUS(make_tmap_2d_bf16(&tq, q, D, p.batch * p.heads_q * p.n, D, 64, BQ));
  IRIS_CHECK_STATUS(make_tmap_2d_bf16(&tk, k, D, p.batch * p.heads_kv * p.n_kv, D, 64, BKV));
  IRIS_CHECK_STATUS(make_tmap_2d_bf16(&tv, v, D, p.batch * p.heads_kv * p.n_kv, D, 64, BKV));
  static bool configured[64] = {false};
  int dev = 0;
  IRIS_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && !configured[dev]) {
    IRIS_CUDA(cudaFuncSetAttribute(flash_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(SMEM_BYTES)));
    configured[dev] = true;
  }
  const int per_cta = TILES * BQ;
  dim3 grid(static_cast<unsigned>((p.n + per_cta - 1) / per_cta), static_cast<unsigned>(p.heads_q),
            static_cast<unsigned>(p.batch));
  flash_attn_kernel<<<grid, THREADS, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_flash_attn_fwd_split(const void* q, const void* k, const void* v, int64_t batch,
                                         int64_t heads_q, int64_t heads_kv, int64_t n, int64_t n_kv,
                                         int64_t head_dim, float scale, float score_bound,
                                         int64_t split, void* o_text, void* o_image, const void* gate_text,
                                         const void* gate_image, int64_t row_stride, void* stream) {
  using namespace iris::attn;
  IRIS_REQUIRE(q && k && v && o_image, "flash_attn_fwd: null pointer");
  IRIS_REQUIRE(head_dim == D, "flash_attn_fwd: head_dim must be 128");
  IRIS_REQUIRE(score_bound >= 0.f && score_bound < INFINITY, "flash_attn_fwd: score_bound must be finite, >= 0");
  IRIS_REQUIRE(batch > 0 && heads_q > 0 && heads_kv > 0 && heads_q % heads_kv == 0,
               "flash_attn_fwd: heads_q must be a positive multiple of heads_kv");
  IRIS_REQUIRE(n > 0 && batch * heads_q * n < (1ll << 31), "flash_attn_fwd: sequence too long");
  IRIS_REQUIRE(n_kv > 0 && batch * heads_kv * n_kv < (1ll << 31), "flash_attn_fwd: key sequence too long");
  IRIS_REQUIRE(split >= 0 && split <= n && (split == 0 || o_text != nullptr), "flash_attn_fwd: bad split");
  IRIS_REQUIRE(row_stride >= heads_q * D && row_stride % 8 == 0, "flash_attn_fwd: o_row_stride");
  IRIS_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o_image) &&
                   (o_text == nullptr || aligned16(o_text)),
               "flash_attn_fwd: alignment");
  IRIS_REQUIRE(split == 0 || (gate_text == nullptr) == (gate_image == nullptr),
               "flash_attn_fwd: gate both streams or neither");
  IRIS_REQUIRE((gate_image == nullptr || aligned16(gate_image)) && (gate_text == nullptr || aligned16(gate_text)),
               "flash_attn_fwd: gate alignment");
  IRIS_REQUIRE(batch <= 65535 && heads_q <= 65535, "flash_attn_fwd: grid too large");
  Params p = {};
  p.batch = batch;
  p.heads_q = heads_q;
  p.heads_kv = heads_kv;
  p.n = n;
  p.n_kv = n_kv;
  p.row_stride = row_stride;
  p.split = split;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.bound_log2 = score_bound * 1.4426950408889634f;
  p.o_text = reinterpret_cast<__nv_bfloat16*>(o_text);
  p.o_image = reinterpret_cast<__nv_bfloat16*>(o_image);
  p.gate_text = reinterpret_cast<const __nv_bfloat16*>(gate_text);
  p.gate_image = reinterpret_cast<const __nv_bfloat16*>(gate_image);
  return launch_attention(q, k, v, p, stream);
}

extern "C" int iris_flash_attn_fwd_peers(const void* q, const void* k, const void* v, int64_t batch, int64_t heads_q,
                                         int64_t heads_kv, int64_t n, int64_t n_kv, int64_t head_dim, float scale,
                                         float score_bound, void* const* o_peers, int world, int64_t tokens_per_rank,
                                         int64_t col0,
                                         int64_t row_stride, void* stream) {
  using namespace iris::attn;
  IRIS_REQUIRE(q && k && v && o_peers, "flash_attn_fwd_peers: null pointer");
  IRIS_REQUIRE(head_dim == D, "flash_attn_fwd_peers: head_dim must be 128");
  IRIS_REQUIRE(score_bound >= 0.f && score_bound < INFINITY, "flash_attn_fwd_peers: score_bound must be finite, >= 0");
  IRIS_REQUIRE(batch > 0 && heads_q > 0 && heads_kv > 0 && heads_q % heads_kv == 0,
               "flash_attn_fwd_peers: heads_q must be a positive multiple of heads_kv");
  IRIS_REQUIRE(world >= 1 && world <= IRIS_MAX_PEERS && tokens_per_rank > 0 && n == world * tokens_per_rank,
               "flash_attn_fwd_peers: n must be world * tokens_per_rank");
  IRIS_REQUIRE(batch * heads_q * n < (1ll << 31) && n_kv > 0 && batch * heads_kv * n_kv < (1ll << 31),
               "flash_attn_fwd_peers: sequence too long");
  IRIS_REQUIRE(col0 >= 0 && col0 % 8 == 0 && row_stride % 8 == 0 && col0 + heads_q * D <= row_stride,
               "flash_attn_fwd_peers: columns col0 + heads_q * 128 must fit a row (multiples of 8)");
  IRIS_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v), "flash_attn_fwd_peers: alignment");
  IRIS_REQUIRE(batch <= 65535 && heads_q <= 65535, "flash_attn_fwd_peers: grid too large");
  Params p = {};
  p.batch = batch;
  p.heads_q = heads_q;
  p.heads_kv = heads_kv;
  p.n = n;
  p.n_kv = n_kv;
  p.row_stride = row_stride;
  p.split = 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.bound_log2 = score_bound * 1.4426950408889634f;
  p.peers = world;
  p.peer_tokens = tokens_per_rank;
  p.peer_col0 = col0;
  p.peer_row_stride = row_stride;
  for (int j = 0; j < world; ++j) {
    IRIS_REQUIRE(o_peers[j] != nullptr && aligned16(o_peers[j]), "flash_attn_fwd_peers: output rows must be aligned");
    p.o_peer[j] = static_cast<__nv_bfloat16*>(o_peers[j]);
  }
  p.o_image = p.o_peer[0];
  return launch_attention(q, k, v, p, stream);
}

extern "C" int iris_flash_attn_fwd(const void* q, const void* k, const void* v, void* o, int64_t batch,
                                   int64_t heads_q, int64_t heads_kv, int64_t n, int64_t head_dim, float scale,
                                   int64_t o_row_stride, void* stream) {
  return iris_flash_attn_fwd_split(q, k, v, batch, heads_q, heads_kv, n, n, head_dim, scale, 0.f, 0, nullptr, o,
                                   nullptr, nullptr, o_row_stride, stream);
}
