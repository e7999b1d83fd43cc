// Persistent, warp-specialised BF16 GEMM on the 5th-generation tensor cores.
//
//   C[m, n] = epilogue( sum_k A[m, k] * W[n, k] )      A: [M, K], W: [N, K], both K-major
//
// This is every Linear of the denoiser step (F.linear in the reference:
// src/iris_metal/model.py:46-52, SwiGLU :51-52, gate :282-283,309, projections
// :284-285,310, pixel stage :332-341). One launch may run up to four
// independent problems (the text- and image-stream projections of a dual
// block, with their own weights): their 128 x 256 output tiles form one
// persistent tile list, so a small problem fills the last wave of a large one.
//
// Per CTA (one per SM, persistent over output tiles of 128 x 256):
//   warp 0      TMA producer: A and W tiles (64-wide K slabs, 128B swizzle)
//               into a 4-stage shared-memory ring;
//   warp 1      TMEM allocator and MMA issuer: one thread issues
//               tcgen05.mma (M=128, N=256, K=16) into one of two TMEM
//               accumulators (2 x 256 fp32 columns) and commits to mbarriers;
//   warps 2..5  epilogue: tcgen05.ld of their 32 TMEM lanes (= 32 rows),
//               fused epilogue math, direct vectorised global stores, then
//               release the accumulator so the next tile's MMAs overlap.
//
// Epilogues: STORE (optional bias, fp32 or bf16 out), ADD (out += acc + bias,
// fp32 residual updated in place), SILU (silu(acc + bias)), SWIGLU (each 256-wide
// W tile holds 128 rows of w1 then the matching 128 rows of w3; writes
// silu(a) * b as bf16, 128 columns per tile), GATE (out = aux * sigmoid(acc),
// bf16), HEADS (two 128-wide [q | k | v] head slots per tile: q and k
// RMS-normed and rotated, all three written to their [b, h, token, 128] or
// head-major layouts). Output and aux rows go through a segmented row map so
// a stream's rows can live inside a joint [text | image] token buffer.
#include <algorithm>

#include "common.cuh"
#include "iris_abi_internal.h"

// 1: batches whose problems all have M >= 256 run on the CTA-pair kernel.
#ifndef IRIS_GEMM_PAIR
#define IRIS_GEMM_PAIR 1
#endif

namespace iris {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 512;        // two 256-column fp32 accumulators
constexpr int THREADS = 192;
constexpr int GROUP_M = 16;           // tile rasterisation: 16 M-blocks per group
constexpr int MAX_PROBLEMS = 4;
// Per epilogue warp, an 8 KB staging tile (32 rows x 256 B) for the peer forms
// of EPI_HEADS: a warp's head rows leave as whole 256-byte rows, two per
// store instruction, instead of 16-byte pieces of 32 different rows, which
// over NVLink would travel as many partial writes.
constexpr int EPI_STAGE_BYTES = 32 * 256;
constexpr int EPI_WARPS = 4;
constexpr size_t SMEM_BYTES =
    1024 /*align slack*/ + STAGES * STAGE_BYTES + 256 /*barriers*/ + EPI_WARPS * EPI_STAGE_BYTES;

enum Epilogue : int { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_GATE = 2, EPI_HEADS = 3, EPI_ADD = 4, EPI_SILU = 5 };

// EPI_HEADS: the tile's 256 columns are two 128-wide head slots of a [q | k |
// v] projection; q and k slots are RMS-normed and rotated, v copied, each to
// its head layout (what iris_qkv_heads does from a stored projection).
// With a peer mode the rows are one sequence-parallel rank's tokens and each
// head row is stored into the buffer of the rank that consumes it (mapped
// into this process), so the projection and the exchange are one kernel.
struct HeadsOut {
  __nv_bfloat16* q;
  __nv_bfloat16* k;
  __nv_bfloat16* v;
  const float* qw;
  const float* kw;
  const float* cos;
  const float* sin;
  float eps;
  int head_major;
  int hq, hkv;
  int64_t tokens, batch, n_out, n_out_kv;
  int peer_mode, world;
  int64_t token_offset, n_dest;
  __nv_bfloat16* q_peer[IRIS_MAX_PEERS];
  __nv_bfloat16* k_peer[IRIS_MAX_PEERS];
  __nv_bfloat16* v_peer[IRIS_MAX_PEERS];
};

struct Problem {
  int M, N, K;
  int num_m, num_n, nk;
  int epilogue;
  int out_dtype;  // 0 f32, 1 bf16
  void* out;
  int64_t ldc;
  RowMap out_map;
  const float* bias;            // [N] or null (STORE only)
  const __nv_bfloat16* aux;     // GATE: [*, ldaux]
  int64_t ldaux;
  RowMap aux_map;
  HeadsOut heads;               // HEADS only
};

struct Batch {
  Problem prob[MAX_PROBLEMS];
  int tile_start[MAX_PROBLEMS + 1];  // prefix sums of the problems' tile counts
  int count;
};

struct TensorMaps {
  CUtensorMap a[MAX_PROBLEMS];
  CUtensorMap b[MAX_PROBLEMS];
};

struct Smem {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t teardown;
  uint32_t tmem_base;
  int abort;
};

static_assert(sizeof(Smem) <= 256, "one-SM barriers must fit their 256-byte slot");
static_assert(SMEM_BYTES <= 232448, "one-SM kernel shared memory");

struct Tile {
  int p, mb, nb;
};

// Tile t of the batch -> (problem, M block, N block); within a problem the
// tiles go in groups of 16 M blocks so concurrent CTAs share A rows and W rows in L2.
IRIS_DEVICE Tile locate(const Batch& bt, int t) {
  int p = 0;
  while (p + 1 < bt.count && t >= bt.tile_start[p + 1]) ++p;
  const Problem& pr = bt.prob[p];
  const int local = t - bt.tile_start[p];
  const int per_group = GROUP_M * pr.num_n;
  const int group = local / per_group;
  const int first_m = group * GROUP_M;
  const int gm = min(GROUP_M, pr.num_m - first_m);
  const int in_group = local - group * per_group;
  return Tile{p, first_m + in_group % gm, in_group / gm};
}

IRIS_DEVICE float sigmoidf_fast(float x) { return 1.0f / (1.0f + __expf(-x)); }

IRIS_DEVICE void store_row32(const Problem& p, int64_t prow, int col0, const float (&v)[32]) {
  if (p.out_dtype == 1) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + prow * p.ldc + col0;
    uint32_t packed[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) packed[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int j = 0; j < 4; ++j) d4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
  } else {
    float4* d4 = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + prow * p.ldc + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
}

// One 128-wide head slot of row m (TMEM columns [col, col + 128) of this
// thread's lane) -> its q / k / v row: RMSNorm over the 128 fp32 accumulators
// times the gain, rotary pairs (2i, 2i+1) by the token's cos / sin, bf16.
// Every lane of the warp runs the TMEM loads (warp-collective); only lanes
// with a real row (`row_ok`) store.
IRIS_DEVICE void store_head_slot(const HeadsOut& hd, uint32_t t_col, int slot, int64_t bn, bool row_ok,
                                 uint8_t* stage) {
  const int64_t b = bn / hd.tokens, t = bn % hd.tokens;
  const bool is_q = slot < hd.hq, is_k = !is_q && slot < hd.hq + hd.hkv;
  const int h = is_q ? slot : is_k ? slot - hd.hq : slot - hd.hq - hd.hkv;
  const int heads = is_q ? hd.hq : hd.hkv;
  const int64_t len = is_q ? hd.n_out : hd.n_out_kv;
  // destinations: one, or (k / v broadcast) one per rank
  const bool scatter = hd.peer_mode == IRIS_HEADS_PEER_SCATTER;
  const bool broadcast = hd.peer_mode == IRIS_HEADS_PEER_BROADCAST_KV && !is_q;
  const int n_dst = broadcast ? hd.world : 1;
  auto dst_of = [&](int j) -> __nv_bfloat16* {
    if (scatter) {
      const int per = heads / hd.world;
      const int owner = h / per;
      __nv_bfloat16* pb = is_q ? hd.q_peer[owner] : is_k ? hd.k_peer[owner] : hd.v_peer[owner];
      return pb + ((b * per + (h - owner * per)) * hd.n_dest + hd.token_offset + t) * 128;
    }
    if (broadcast) return (is_k ? hd.k_peer[j] : hd.v_peer[j]) + ((b * heads + h) * hd.n_dest + hd.token_offset + t) * 128;
    __nv_bfloat16* base = is_q ? hd.q : is_k ? hd.k : hd.v;
    return base + ((hd.head_major ? h * hd.batch + b : b * heads + h) * len + t) * 128;
  };
  float inv = 1.f;
  const float* gain = is_q ? hd.qw : hd.kw;
  if (is_q || is_k) {
    float ss = 0.f;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      tmem_ld32(t_col + c * 32, r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) ss = fmaf(__uint_as_float(r[j]), __uint_as_float(r[j]), ss);
    }
    inv = rsqrtf(ss * (1.f / 128.f) + hd.eps);
  }
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t r[32];
    tmem_ld32(t_col + c * 32, r);
    tmem_wait_ld();
    uint32_t packed[16];
    if (is_q || is_k) {
      const float4* g4 = reinterpret_cast<const float4*>(gain + c * 32);
      const float4* c4 = reinterpret_cast<const float4*>(hd.cos + t * 64 + c * 16);
      const float4* s4 = reinterpret_cast<const float4*>(hd.sin + t * 64 + c * 16);
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {  // 8 columns = 4 rotary pairs at a time
        const float4 ga = __ldg(g4 + 2 * q4), gb = __ldg(g4 + 2 * q4 + 1);
        const float4 cs = __ldg(c4 + q4), sn = __ldg(s4 + q4);
        const float g[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
        const float cc[4] = {cs.x, cs.y, cs.z, cs.w}, sc[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = q4 * 8 + 2 * e;
          const float a = __uint_as_float(r[j]) * inv * g[2 * e];
          const float bb = __uint_as_float(r[j + 1]) * inv * g[2 * e + 1];
          packed[q4 * 4 + e] = pack_bf16x2(a * cc[e] - bb * sc[e], a * sc[e] + bb * cc[e]);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) packed[j] = pack_bf16x2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
    }
    if (hd.peer_mode != IRIS_HEADS_LOCAL) {
      // 16-byte chunk q of row r at (q ^ (r & 15)) * 16: the 32 rows' same chunk spread over the banks
      const int r = threadIdx.x & 31;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(stage + r * 256 + (((c * 4 + j) ^ (r & 15)) * 16)) =
            make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
    } else if (row_ok) {
      uint4* d4 = reinterpret_cast<uint4*>(dst_of(0) + c * 32);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        d4[j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
    }
  }
  if (hd.peer_mode == IRIS_HEADS_LOCAL) return;
  // write-out: lane L stores 16-byte chunk L % 16 of row 2k + L / 16, so each
  // instruction writes two whole 256-byte rows (each row's destination and
  // validity come from the thread that owns it)
  __syncwarp();
  const int lane = threadIdx.x & 31;
#pragma unroll 1
  for (int r_dst = 0; r_dst < n_dst; ++r_dst) {
    const unsigned long long mine = row_ok ? reinterpret_cast<unsigned long long>(dst_of(r_dst)) : 0ull;
#pragma unroll 4
    for (int k = 0; k < 16; ++k) {
      const int row = 2 * k + (lane >> 4), q = lane & 15;
      const unsigned long long dst = __shfl_sync(0xffffffffu, mine, row);
      if (dst != 0ull)
        *reinterpret_cast<uint4*>(dst + q * 16) =
            *reinterpret_cast<const uint4*>(stage + row * 256 + ((q ^ (row & 15)) * 16));
    }
  }
  __syncwarp();  // the tile is reused by this warp's next head slot
}

// The epilogue of one accumulator tile for this thread's row m (TMEM lane
// base `t_base`, column 0 of the accumulator); `nb` is the tile's N block.
IRIS_DEVICE void epilogue_row(const Problem& p, uint32_t t_base, int64_t m, int nb, uint8_t* stage) {
  const bool row_ok = m < p.M;
  if (p.epilogue == EPI_HEADS) {
    const int64_t bn = row_ok ? p.out_map(m) : 0;
    const int slots = p.heads.hq + 2 * p.heads.hkv;
#pragma unroll 1
    for (int k = 0; k < 2; ++k) {
      const int slot = nb * 2 + k;  // uniform across the warp, as the TMEM loads require
      if (slot < slots) store_head_slot(p.heads, t_base + k * 128, slot, bn, row_ok, stage);
    }
    return;
  }
  if (p.epilogue == EPI_SWIGLU) {
    const int64_t prow = row_ok ? p.out_map(m) : 0;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t ra[32], rb[32];
      tmem_ld32(t_base + c * 32, ra);
      tmem_ld32(t_base + 128 + c * 32, rb);
      tmem_wait_ld();
      const int col0 = nb * (BN / 2) + c * 32;
      if (row_ok && col0 < p.N / 2) {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float a = __uint_as_float(ra[j]);
          v[j] = a * sigmoidf_fast(a) * __uint_as_float(rb[j]);
        }
        store_row32(p, prow, col0, v);
      }
    }
    return;
  }
  const int64_t prow = row_ok ? p.out_map(m) : 0;
  const int64_t arow = (row_ok && p.epilogue == EPI_GATE) ? p.aux_map(m) : 0;
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    uint32_t r[32];
    tmem_ld32(t_base + c * 32, r);
    tmem_wait_ld();
    const int col0 = nb * BN + c * 32;
    if (row_ok && col0 < p.N) {
      float v[32];
      if (p.epilogue == EPI_GATE) {
        const uint4* a4 = reinterpret_cast<const uint4*>(p.aux + arow * p.ldaux + col0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 w = a4[j];
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float2 f = unpack_bf16x2(ws[h]);
            const int e = j * 8 + h * 2;
            v[e] = f.x * sigmoidf_fast(__uint_as_float(r[e]));
            v[e + 1] = f.y * sigmoidf_fast(__uint_as_float(r[e + 1]));
          }
        }
      } else {
        if (p.bias != nullptr) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) + __ldg(p.bias + col0 + j);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        }
        if (p.epilogue == EPI_SILU) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = v[j] * sigmoidf_fast(v[j]);
        } else if (p.epilogue == EPI_ADD) {  // residual update in place (f32 out only)
          const float4* o4 = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.out) + prow * p.ldc + col0);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 o = o4[j];
            v[4 * j] += o.x;
            v[4 * j + 1] += o.y;
            v[4 * j + 2] += o.z;
            v[4 * j + 3] += o.w;
          }
        }
      }
      store_row32(p, prow, col0, v);
    }
  }
}

__global__ void __launch_bounds__(THREADS, 1)
    gemm_bf16_kernel(const __grid_constant__ TensorMaps maps, const __grid_constant__ Batch bt) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzled tiles
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = base;
  Smem* s = reinterpret_cast<Smem*>(base + STAGES * STAGE_BYTES);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_tiles = bt.tile_start[bt.count];

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s->full[i], 1);
      mbar_init(&s->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s->tmem_full[i], 1);
      mbar_init(&s->tmem_empty[i], 4);
    }
    mbar_init(&s->teardown, 1);
    s->abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    for (int p = 0; p < bt.count; ++p) {
      tma_prefetch_desc(&maps.a[p]);
      tma_prefetch_desc(&maps.b[p]);
    }
  }
  if (warp == 1) tmem_alloc(&s->tmem_base, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s->tmem_base;
  volatile int* abort = &s->abort;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued_phase[STAGES];
#pragma unroll
      for (int i = 0; i < STAGES; ++i) issued_phase[i] = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const Tile tl = locate(bt, t);
        const CUtensorMap* ma = &maps.a[tl.p];
        const CUtensorMap* mw = &maps.b[tl.p];
        const int nk = bt.prob[tl.p].nk;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&s->empty[stage], phase ^ 1u, abort)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = tiles + stage * STAGE_BYTES;
          uint8_t* b_dst = a_dst + A_BYTES;
          mbar_arrive_expect_tx(&s->full[stage], STAGE_BYTES);
          tma_load_2d(ma, &s->full[stage], a_dst, kb * BK, tl.mb * BM);
          tma_load_2d(mw, &s->full[stage], b_dst, kb * BK, tl.nb * BN);
          issued_phase[stage] = static_cast<int>(phase);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // let the copies already in flight land before shared memory is released
        int dummy = 0;
        for (int i = 0; i < STAGES; ++i)
          if (issued_phase[i] >= 0) mbar_wait(&s->full[i], static_cast<uint32_t>(issued_phase[i]), &dummy);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
        const int nk = bt.prob[locate(bt, t).p].nk;
        const int acc = it & 1;
        const uint32_t acc_phase = static_cast<uint32_t>((it >> 1) & 1);
        if (!mbar_wait(&s->tmem_empty[acc], acc_phase ^ 1u, abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&s->full[stage], phase, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_addr(tiles + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = umma_desc(a_addr + k * 32, 16, 1024, kLayoutSw128);
            const uint64_t bd = umma_desc(b_addr + k * 32, 16, 1024, kLayoutSw128);
            umma_ss(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&s->empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(&s->tmem_full[acc]);
      }
      // all MMAs of this thread are complete once this barrier flips
      umma_commit(&s->teardown);
      int dummy = 0;
      mbar_wait(&s->teardown, 0, &dummy);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
    const int row_in_tile = quarter * 32 + lane;
    uint8_t* stage = base + STAGES * STAGE_BYTES + 256 + (warp - 2) * EPI_STAGE_BYTES;
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
      const Tile tl = locate(bt, t);
      const Problem& p = bt.prob[tl.p];
      const int acc = it & 1;
      const uint32_t acc_phase = static_cast<uint32_t>((it >> 1) & 1);
      // warp-uniform decision: tcgen05.ld below is a .sync.aligned warp instruction
      if (!__all_sync(0xffffffffu, mbar_wait(&s->tmem_full[acc], acc_phase, abort))) break;
      tc_fence_after();
      const uint32_t t_base = tmem + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
      epilogue_row(p, t_base, static_cast<int64_t>(tl.mb) * BM + row_in_tile, tl.nb, stage);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s->tmem_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// ---------------------------------------------------------------------------
// CTA-pair form (cta_group::2): a cluster of two CTAs on paired SMs computes a
// 256 x 256 tile. Each CTA TMA-loads its own 128 rows of A and its half (128
// rows) of the W tile, 32 KB per 64-wide K slab, into a 6-stage ring. Both
// CTAs' copies complete on the leader CTA's "full" barrier, whose byte count
// the leader's producer alone announces for the pair (a remote arrive from the
// peer's producer on every slab halved the kernel's rate). The leader's
// MMA thread issues tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16), which
// reads A and W from both CTAs' shared memory and writes each CTA's 128 rows x
// 256 fp32 columns into that CTA's TMEM; its commits are sent to each CTA's
// barrier separately. Both CTAs run the same epilogue on their own rows; the
// peer's epilogue warps release an accumulator with remote arrivals on the
// leader's barrier. Per SM this halves the W bytes each k-slab brings in.
namespace pair {
constexpr int BM = 256;  // pair tile rows, 128 per CTA
constexpr int STAGES = 6;
constexpr int A_BYTES = 128 * BK * 2;  // 16 KB: this CTA's rows
constexpr int B_BYTES = 128 * BK * 2;  // 16 KB: this CTA's half of the W tile
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr size_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256 + EPI_WARPS * EPI_STAGE_BYTES;

struct Smem {
  uint64_t full[STAGES];  // used in the leader only: both CTAs' copies complete here
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];  // used in the leader only: 4 local + 4 peer epilogue warps
  uint64_t teardown;
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Smem) <= 256, "pair barriers must fit their 256-byte slot");
static_assert(SMEM_BYTES <= 232448, "pair kernel shared memory");
}  // namespace pair

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ TensorMaps maps, const __grid_constant__ Batch bt) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = base;
  pair::Smem* s = reinterpret_cast<pair::Smem*>(base + pair::STAGES * pair::STAGE_BYTES);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int num_tiles = bt.tile_start[bt.count];
  const int pair_id = blockIdx.x / 2;
  const int pairs = gridDim.x / 2;

  if (threadIdx.x == 0) {
    for (int i = 0; i < pair::STAGES; ++i) {
      mbar_init(&s->full[i], 1);
      mbar_init(&s->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s->tmem_full[i], 1);
      mbar_init(&s->tmem_empty[i], 8);
    }
    mbar_init(&s->teardown, 1);
    s->abort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    for (int p = 0; p < bt.count; ++p) {
      tma_prefetch_desc(&maps.a[p]);
      tma_prefetch_desc(&maps.b[p]);
    }
  }
  if (warp == 1) tmem_alloc_pair(&s->tmem_base, TMEM_COLS);
  tc_fence_before();
  cluster_sync();  // every barrier of both CTAs exists before any remote arrival
  tc_fence_after();
  const uint32_t tmem = s->tmem_base;
  volatile int* abort = &s->abort;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int t = pair_id; t < num_tiles && ok; t += pairs) {
        const Tile tl = locate(bt, t);
        const CUtensorMap* ma = &maps.a[tl.p];
        const CUtensorMap* mw = &maps.b[tl.p];
        const int nk = bt.prob[tl.p].nk;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&s->empty[stage], phase ^ 1u, abort)) {
            ok = false;
            break;
          }
          const uint32_t full_leader = map_to_cta(&s->full[stage], 0);
          uint8_t* a_dst = tiles + stage * pair::STAGE_BYTES;
          uint8_t* b_dst = a_dst + pair::A_BYTES;
          // The leader announces both CTAs' bytes; the peer's copies may land
          // first (the transaction count dips below zero until it does).
          if (leader) mbar_arrive_expect_tx(&s->full[stage], 2 * pair::STAGE_BYTES);
          tma_load_2d_pair(ma, full_leader, a_dst, kb * BK, tl.mb * pair::BM + static_cast<int>(rank) * 128);
          tma_load_2d_pair(mw, full_leader, b_dst, kb * BK, tl.nb * BN + static_cast<int>(rank) * 128);
          ++issued;
          if (++stage == pair::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && issued > 0) {
        // the loads in flight target both CTAs' shared memory: give them time to land
        const uint64_t t0 = global_timer_ns();
        while (global_timer_ns() - t0 < 1000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && leader) {
      const uint32_t idesc = idesc_bf16_f32(pair::BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = pair_id; t < num_tiles && ok; t += pairs, ++it) {
        const int nk = bt.prob[locate(bt, t).p].nk;
        const int acc = it & 1;
        const uint32_t acc_phase = static_cast<uint32_t>((it >> 1) & 1);
        if (!mbar_wait_cluster(&s->tmem_empty[acc], acc_phase ^ 1u, abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&s->full[stage], phase, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_addr(tiles + stage * pair::STAGE_BYTES);
          const uint32_t b_addr = a_addr + pair::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = umma_desc(a_addr + k * 32, 16, 1024, kLayoutSw128);
            const uint64_t bd = umma_desc(b_addr + k * 32, 16, 1024, kLayoutSw128);
            umma_ss_pair(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(map_to_cta(&s->empty[stage], 0));
          umma_commit_pair(map_to_cta(&s->empty[stage], 1));
          if (++stage == pair::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) {
          umma_commit_pair(map_to_cta(&s->tmem_full[acc], 0));
          umma_commit_pair(map_to_cta(&s->tmem_full[acc], 1));
        }
      }
      umma_commit_pair(map_to_cta(&s->teardown, 0));
      int dummy = 0;
      mbar_wait(&s->teardown, 0, &dummy);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    uint8_t* stage = base + pair::STAGES * pair::STAGE_BYTES + 256 + (warp - 2) * EPI_STAGE_BYTES;
    const uint32_t empty_leader = map_to_cta(&s->tmem_empty[0], 0);
    int it = 0;
    for (int t = pair_id; t < num_tiles; t += pairs, ++it) {
      const Tile tl = locate(bt, t);
      const Problem& p = bt.prob[tl.p];
      const int acc = it & 1;
      const uint32_t acc_phase = static_cast<uint32_t>((it >> 1) & 1);
      if (!__all_sync(0xffffffffu, mbar_wait_cluster(&s->tmem_full[acc], acc_phase, abort))) break;
      tc_fence_after();
      const uint32_t t_base = tmem + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
      epilogue_row(p, t_base, static_cast<int64_t>(tl.mb) * pair::BM + static_cast<int64_t>(rank) * 128 + row_in_tile,
                   tl.nb, stage);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(empty_leader + static_cast<uint32_t>(acc) * 8u);
    }
  }

  tc_fence_before();
  cluster_sync();  // no CTA leaves while the other may still address its barriers or TMEM
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, TMEM_COLS);
}

int check_heads(const iris_gemm_problem& q) {
  const iris_heads_epilogue* hd = q.heads;
  IRIS_REQUIRE(hd != nullptr, "iris_gemm_bf16: the heads epilogue needs its parameters");
  IRIS_REQUIRE(hd->heads_q > 0 && hd->heads_kv >= 0 && q.N == (hd->heads_q + 2 * hd->heads_kv) * 128,
               "iris_gemm_bf16: heads epilogue needs N = (heads_q + 2 heads_kv) * 128");
  const int mode = hd->peer_mode;
  IRIS_REQUIRE(mode == IRIS_HEADS_LOCAL || mode == IRIS_HEADS_PEER_SCATTER || mode == IRIS_HEADS_PEER_BROADCAST_KV,
               "iris_gemm_bf16: unknown heads peer_mode");
  IRIS_REQUIRE(hd->q_weight && hd->cos && hd->sin && (hd->heads_kv == 0 || hd->k_weight),
               "iris_gemm_bf16: heads epilogue null pointer");
  IRIS_REQUIRE(aligned16(hd->q_weight) && aligned16(hd->cos) && aligned16(hd->sin) &&
                   (hd->heads_kv == 0 || aligned16(hd->k_weight)),
               "iris_gemm_bf16: heads epilogue pointers must be 16-byte aligned");
  const bool local_q = mode != IRIS_HEADS_PEER_SCATTER, local_kv = mode == IRIS_HEADS_LOCAL;
  IRIS_REQUIRE(!local_q || (hd->q_out && aligned16(hd->q_out)), "iris_gemm_bf16: heads epilogue q_out");
  IRIS_REQUIRE(!local_kv || hd->heads_kv == 0 || (hd->k_out && hd->v_out && aligned16(hd->k_out) && aligned16(hd->v_out)),
               "iris_gemm_bf16: heads epilogue k_out / v_out");
  if (mode != IRIS_HEADS_LOCAL) {
    IRIS_REQUIRE(hd->world >= 1 && hd->world <= IRIS_MAX_PEERS, "iris_gemm_bf16: heads epilogue world out of range");
    IRIS_REQUIRE(hd->token_offset >= 0 && hd->token_offset + hd->tokens <= hd->n_dest,
                 "iris_gemm_bf16: heads epilogue token_offset + tokens > n_dest");
    if (mode == IRIS_HEADS_PEER_SCATTER)
      IRIS_REQUIRE(hd->heads_q % hd->world == 0 && hd->heads_kv % hd->world == 0,
                   "iris_gemm_bf16: scattered heads must divide over the ranks");
    for (int j = 0; j < hd->world; ++j) {
      const bool q_ok = mode != IRIS_HEADS_PEER_SCATTER || (hd->q_peer[j] && aligned16(hd->q_peer[j]));
      const bool kv_ok = hd->heads_kv == 0 || (hd->k_peer[j] && hd->v_peer[j] && aligned16(hd->k_peer[j]) &&
                                               aligned16(hd->v_peer[j]));
      IRIS_REQUIRE(q_ok && kv_ok, "iris_gemm_bf16: heads epilogue peer buffers must be non-null and 16-byte aligned");
    }
  }
  IRIS_REQUIRE(hd->tokens > 0 && hd->batch > 0 && (!local_q || hd->tokens <= hd->n_out) &&
                   (!local_kv || hd->heads_kv == 0 || hd->tokens <= hd->n_out_kv),
               "iris_gemm_bf16: heads epilogue needs tokens <= n_out, n_out_kv");
  // the largest row the map produces must stay inside batch * tokens positions
  const int64_t last = (q.M - 1) / q.out_seg_rows * q.out_seg_stride + q.out_seg_offset +
                       std::min<int64_t>(q.out_seg_rows, q.M) - 1;
  IRIS_REQUIRE(q.out_seg_stride >= 0 && q.out_seg_offset >= 0 && last < hd->batch * hd->tokens,
               "iris_gemm_bf16: heads epilogue row map leaves the batch * tokens positions");
  return IRIS_OK;
}

int check_problem(const iris_gemm_problem& q) {
  if (q.epilogue == EPI_HEADS) {
    IRIS_REQUIRE(q.a && q.w, "iris_gemm_bf16: null pointer");
  } else {
    IRIS_REQUIRE(q.a && q.w && q.out, "iris_gemm_bf16: null pointer");
  }
  IRIS_REQUIRE(q.M > 0 && q.N > 0 && q.K > 0, "iris_gemm_bf16: empty problem");
  IRIS_REQUIRE(q.M < (1ll << 31) && q.N < (1ll << 31) && q.K < (1ll << 31), "iris_gemm_bf16: dimension too large");
  IRIS_REQUIRE(q.K % 8 == 0 && q.lda % 8 == 0 && q.ldw % 8 == 0 && q.lda >= q.K && q.ldw >= q.K,
               "iris_gemm_bf16: K and leading dimensions must be multiples of 8 (16-byte TMA rows)");
  IRIS_REQUIRE(q.N % 32 == 0, "iris_gemm_bf16: N must be a multiple of 32");
  IRIS_REQUIRE(q.epilogue >= EPI_STORE && q.epilogue <= EPI_SILU, "iris_gemm_bf16: unknown epilogue");
  IRIS_REQUIRE(q.out_seg_rows > 0 && q.aux_seg_rows > 0, "iris_gemm_bf16: row maps need seg_rows > 0");
  IRIS_REQUIRE(aligned16(q.a) && aligned16(q.w), "iris_gemm_bf16: pointers must be 16-byte aligned");
  if (q.epilogue == EPI_HEADS) return check_heads(q);
  IRIS_REQUIRE(q.out_dtype == 0 || q.out_dtype == 1, "iris_gemm_bf16: out dtype must be f32 or bf16");
  IRIS_REQUIRE(aligned16(q.out), "iris_gemm_bf16: pointers must be 16-byte aligned");
  IRIS_REQUIRE(q.ldc % 8 == 0, "iris_gemm_bf16: ldc must be a multiple of 8");
  if (q.epilogue == EPI_SWIGLU) {
    IRIS_REQUIRE(q.N % BN == 0 && q.out_dtype == 1 && q.ldc >= q.N / 2,
                 "iris_gemm_bf16: SwiGLU needs N % 256 == 0 (paired 128-row w1/w3 blocks) and bf16 out");
  } else {
    IRIS_REQUIRE(q.ldc >= q.N, "iris_gemm_bf16: ldc < N");
  }
  if (q.epilogue == EPI_ADD)
    IRIS_REQUIRE(q.out_dtype == 0, "iris_gemm_bf16: the add epilogue updates an f32 output in place");
  if (q.epilogue == EPI_GATE) {
    IRIS_REQUIRE(q.aux != nullptr && aligned16(q.aux) && q.ldaux % 8 == 0 && q.ldaux >= q.N && q.out_dtype == 1,
                 "iris_gemm_bf16: gate epilogue needs an aligned bf16 aux with ldaux % 8 == 0");
    IRIS_REQUIRE(q.bias == nullptr, "iris_gemm_bf16: gate epilogue takes no bias");
  }
  return IRIS_OK;
}

}  // namespace gemm
}  // namespace iris

using namespace iris;

extern "C" int iris_gemm_bf16_grouped(const iris_gemm_problem* problems, int count, void* stream) {
  using namespace iris::gemm;
  IRIS_REQUIRE(problems != nullptr && count >= 1 && count <= MAX_PROBLEMS,
               "iris_gemm_bf16_grouped: 1 to 4 problems per launch");
  // The CTA-pair kernel runs a batch whose every problem fills at least one
  // 256-row pair tile; smaller problems keep the one-SM kernel.
  bool use_pair = IRIS_GEMM_PAIR != 0;
  for (int i = 0; i < count; ++i) use_pair = use_pair && problems[i].M >= pair::BM;
  const int bm = use_pair ? pair::BM : BM;
  const int w_box_rows = use_pair ? BN / 2 : BN;
  TensorMaps maps;
  Batch bt;
  bt.count = count;
  bt.tile_start[0] = 0;
  int64_t total = 0;
  for (int i = 0; i < count; ++i) {
    const iris_gemm_problem& q = problems[i];
    IRIS_CHECK_STATUS(check_problem(q));
    IRIS_CHECK_STATUS(make_tmap_2d_bf16(&maps.a[i], q.a, q.K, q.M, q.lda, BK, BM));
    IRIS_CHECK_STATUS(make_tmap_2d_bf16(&maps.b[i], q.w, q.K, q.N, q.ldw, BK, w_box_rows));
    Problem& p = bt.prob[i];
    p.M = static_cast<int>(q.M);
    p.N = static_cast<int>(q.N);
    p.K = static_cast<int>(q.K);
    p.num_m = static_cast<int>((q.M + bm - 1) / bm);
    p.num_n = static_cast<int>((q.N + BN - 1) / BN);
    p.nk = static_cast<int>((q.K + BK - 1) / BK);
    p.epilogue = q.epilogue;
    p.out_dtype = q.out_dtype;
    p.out = q.out;
    p.ldc = q.ldc;
    p.out_map = RowMap{q.out_seg_rows, q.out_seg_stride, q.out_seg_offset};
    p.bias = q.bias;
    p.aux = reinterpret_cast<const __nv_bfloat16*>(q.aux);
    p.ldaux = q.ldaux;
    p.aux_map = RowMap{q.aux_seg_rows, q.aux_seg_stride, q.aux_seg_offset};
    p.heads = HeadsOut{};
    if (q.epilogue == EPI_HEADS) {
      const iris_heads_epilogue& hd = *q.heads;
      HeadsOut& ho = p.heads;
      ho.q = static_cast<__nv_bfloat16*>(hd.q_out);
      ho.k = static_cast<__nv_bfloat16*>(hd.k_out);
      ho.v = static_cast<__nv_bfloat16*>(hd.v_out);
      ho.qw = hd.q_weight;
      ho.kw = hd.k_weight;
      ho.cos = hd.cos;
      ho.sin = hd.sin;
      ho.eps = hd.eps;
      ho.head_major = hd.head_major;
      ho.hq = static_cast<int>(hd.heads_q);
      ho.hkv = static_cast<int>(hd.heads_kv);
      ho.tokens = hd.tokens;
      ho.batch = hd.batch;
      ho.n_out = hd.n_out;
      ho.n_out_kv = hd.n_out_kv;
      ho.peer_mode = hd.peer_mode;
      ho.world = hd.world;
      ho.token_offset = hd.token_offset;
      ho.n_dest = hd.n_dest;
      for (int j = 0; j < IRIS_MAX_PEERS; ++j) {
        const bool used = j < hd.world;
        ho.q_peer[j] = used ? static_cast<__nv_bfloat16*>(hd.q_peer[j]) : nullptr;
        ho.k_peer[j] = used ? static_cast<__nv_bfloat16*>(hd.k_peer[j]) : nullptr;
        ho.v_peer[j] = used ? static_cast<__nv_bfloat16*>(hd.v_peer[j]) : nullptr;
      }
    }
    total += static_cast<int64_t>(p.num_m) * p.num_n;
    IRIS_REQUIRE(total < (1ll << 30), "iris_gemm_bf16_grouped: too many tiles");
    bt.tile_start[i + 1] = static_cast<int>(total);
  }
  static bool configured[64] = {false};
  int dev = 0;
  IRIS_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && !configured[dev]) {
    IRIS_CUDA(cudaFuncSetAttribute(gemm_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(SMEM_BYTES)));
    IRIS_CUDA(cudaFuncSetAttribute(gemm_bf16_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(pair::SMEM_BYTES)));
    configured[dev] = true;
  }
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (use_pair) {
    // Not every SM has a partner SM that a cluster of two can use: size the
    // persistent grid to the clusters that are resident at once, or the tiles
    // of the clusters left over would run as a second wave.
    static int resident_pairs[64] = {0};
    int limit = dev < 64 ? resident_pairs[dev] : 0;
    if (limit == 0) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(num_sms()));
      cfg.blockDim = dim3(THREADS);
      cfg.dynamicSmemBytes = pair::SMEM_BYTES;
      IRIS_CUDA(cudaOccupancyMaxActiveClusters(&limit, gemm_bf16_pair_kernel, &cfg));
      IRIS_REQUIRE(limit > 0, "iris_gemm_bf16_grouped: no CTA pair fits on this device");
      if (dev < 64) resident_pairs[dev] = limit;
    }
    const int pairs = total < limit ? static_cast<int>(total) : limit;
    gemm_bf16_pair_kernel<<<2 * pairs, THREADS, pair::SMEM_BYTES, st>>>(maps, bt);
  } else {
    const int grid = total < num_sms() ? static_cast<int>(total) : num_sms();
    gemm_bf16_kernel<<<grid, THREADS, SMEM_BYTES, st>>>(maps, bt);
  }
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}

extern "C" int iris_gemm_bf16(const void* a, int64_t lda, const void* w, int64_t ldw, void* out, int out_dtype,
                              int64_t ldc, int64_t M, int64_t N, int64_t K, int epilogue, const float* bias,
                              const void* aux, int64_t ldaux, int64_t out_seg_rows, int64_t out_seg_stride,
                              int64_t out_seg_offset, int64_t aux_seg_rows, int64_t aux_seg_stride,
                              int64_t aux_seg_offset, void* stream) {
  iris_gemm_problem q;
  q.a = a;
  q.lda = lda;
  q.w = w;
  q.ldw = ldw;
  q.out = out;
  q.out_dtype = out_dtype;
  q.ldc = ldc;
  q.M = M;
  q.N = N;
  q.K = K;
  q.epilogue = epilogue;
  q.bias = bias;
  q.aux = aux;
  q.ldaux = ldaux;
  q.out_seg_rows = out_seg_rows;
  q.out_seg_stride = out_seg_stride;
  q.out_seg_offset = out_seg_offset;
  q.aux_seg_rows = aux_seg_rows;
  q.aux_seg_stride = aux_seg_stride;
  q.aux_seg_offset = aux_seg_offset;
  q.heads = nullptr;
  IRIS_REQUIRE(epilogue != iris::gemm::EPI_HEADS, "iris_gemm_bf16: the heads epilogue runs through iris_gemm_bf16_grouped");
  return iris_gemm_bf16_grouped(&q, 1, stream);
}
