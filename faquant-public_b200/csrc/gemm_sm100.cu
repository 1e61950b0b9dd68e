// K3 -- bf16 GEMM y = a . b^T (+ bias) on the 5th-generation tensor cores.
//
// The W4A4 Linear runs its GEMM on the exactly-dequantized HiF4 operands in bf16:
// every HiF4 value has at most 6 significant bits, so bf16 holds it exactly,
// products are exact and the fp32 accumulation is the reference's fake-quant
// semantics (F.linear on the QDQ tensors, quantization.py:277). No block-scaled
// FP4/FP8 MMA represents HiF4 exactly: E2M1 lacks the 1.25/1.75 element steps
// and the E6M2 scale mantissa cannot be a UE8M0 block scale.
//
// Structure (one CTA per SM, persistent over 128x256 output tiles):
//   warp 0      TMA producer: A [128 x 64] and B [256 x 64] bf16 tiles, 128-byte
//               swizzle, into a 4-stage shared-memory ring (48 KB per stage);
//   warp 1      allocates 512 TMEM columns; one lane issues tcgen05.mma
//               (M=128, N=256, K=16, kind::f16) and tcgen05.commit;
//   warps 2..5  epilogue: tcgen05.ld of the fp32 accumulator (one row per
//               thread), bias, bf16 rounding, 16-byte stores.
// The two accumulators (2 x 256 columns) let the epilogue of tile i overlap the
// main loop of tile i+1. Every wait is bounded (common.cuh, mbar_wait).
#include <algorithm>
#include <atomic>
#include <cstdlib>

#include "common.cuh"
#include "tma.h"

namespace faq {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = 512;
constexpr int THREADS = 192;
constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN, false, false);
constexpr size_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;

struct Params {
  int m, n, k;
  int tiles_m, tiles_n, kblocks;
  int group_m;  // M tiles per group of the L2-friendly tile order
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual;  // [m, ldr] added to the bf16 product, or null
  int64_t ldr;
  __nv_bfloat16* y;
  int64_t ldy;
  bool y_vec;
  bool r_vec;
};

// Tile order: groups of group_m M-tiles; inside a group the M tile varies fastest and
// the group sweeps all N tiles. A wave of 148 CTAs then reads group_m A panels and about
// 148 / group_m B panels, instead of every A panel (the plain M-fastest order, whose A
// re-reads from DRAM once per wave are the dominant traffic when A outgrows a die's L2).
__device__ __forceinline__ void tile_coords(const Params& p, int tile, int& tm, int& tn) {
  const int per_group = p.group_m * p.tiles_n;
  const int group = tile / per_group, in_group = tile - group * per_group;
  const int first_m = group * p.group_m;
  const int rows = min(p.group_m, p.tiles_m - first_m);
  tm = first_m + in_group % rows;
  tn = in_group / rows;
}

// Output values of a 32-column run of one row: fl(acc + bias), and with a residual
// fl(bf16(fl(acc + bias)) + residual) -- the bf16 product first rounded, then the bf16 add
// of eager `residual + linear(x)`, so the fused epilogue gives the same bits as the two
// separate steps.
__device__ __forceinline__ void store_row32(const Params& p, int row, int col, const float (&v)[32]) {
  if (row >= p.m || col >= p.n) return;
  float r[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float b = 0.0f;
    if (p.bias != nullptr && col + i < p.n) b = __bfloat162float(p.bias[col + i]);
    r[i] = v[i] + b;
  }
  if (p.residual != nullptr) {
    const __nv_bfloat16* res = p.residual + static_cast<int64_t>(row) * p.ldr + col;
    if (p.r_vec && col + 32 <= p.n) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 w = reinterpret_cast<const uint4*>(res)[j];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const int i = 8 * j + 2 * h;
          r[i] = bf16_round(r[i]) + __uint_as_float(ws[h] << 16);
          r[i + 1] = bf16_round(r[i + 1]) + __uint_as_float(ws[h] & 0xFFFF0000u);
        }
      }
    } else {
      for (int i = 0; i < 32 && col + i < p.n; ++i) r[i] = bf16_round(r[i]) + __bfloat162float(res[i]);
    }
  }
  __nv_bfloat16* dst = p.y + static_cast<int64_t>(row) * p.ldy + col;
  if (p.y_vec && col + 32 <= p.n) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t w[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const __nv_bfloat162 pair = __floats2bfloat162_rn(r[8 * j + 2 * h], r[8 * j + 2 * h + 1]);
        w[h] = *reinterpret_cast<const uint32_t*>(&pair);
      }
      d4[j] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
    for (int i = 0; i < 32 && col + i < p.n; ++i) dst[i] = __float2bfloat16_rn(r[i]);
  }
}

__global__ void __launch_bounds__(THREADS, 1)
    gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = base + STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + STAGES * STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = bars + 2 * STAGES + NUM_ACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 2 * NUM_ACC);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), 1);
    }
    for (int a = 0; a < NUM_ACC; ++a) {
      mbar_init(smem_addr(&tfull[a]), 1);
      mbar_init(smem_addr(&tempty[a]), 4);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = p.tiles_m * p.tiles_n;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int tm, tn;
        tile_coords(p, tile, tm, tn);
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait_site(smem_addr(&empty[stage]), phase ^ 1, 21, kb)) { ok = false; break; }
          mbar_arrive_expect_tx(smem_addr(&full[stage]), STAGE_BYTES);
          tma_load_2d(smem_addr(sA + stage * A_BYTES), &tmap_a, smem_addr(&full[stage]), kb * BK, tm * BM);
          tma_load_2d(smem_addr(sB + stage * B_BYTES), &tmap_b, smem_addr(&full[stage]), kb * BK, tn * BN);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // drain: wait (bounded) until the tensor cores released every loaded stage
      for (int s = 0; s < STAGES && ok; ++s) {
        if (!mbar_wait_site(smem_addr(&empty[stage]), phase ^ 1, 22, s)) break;
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait_site(smem_addr(&tempty[acc]), acc_phase ^ 1, 23, it)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait_site(smem_addr(&full[stage]), phase, 24, kb)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_addr(sA + stage * A_BYTES), b0 = smem_addr(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            tc_mma_f16(d_tmem, sw128_kmajor_desc(a0 + kk * 32), sw128_kmajor_desc(b0 + kk * 32), IDESC,
                       (kb | kk) != 0);
          tc_commit(smem_addr(&empty[stage]));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        tc_commit(smem_addr(&tfull[acc]));
      }
    }
    __syncwarp();
  } else {
    const int quarter = warp & 3;
    int it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait_warp(smem_addr(&tfull[acc]), acc_phase, 25, it)) break;
      tc_fence_after();
      int tm, tn;
      tile_coords(p, tile, tm, tn);
      const int row = tm * BM + quarter * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld32(taddr + c, r);
        tc_wait_ld();
        reg_fence32(r);
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        store_row32(p, row, tn * BN + c, v);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&tempty[acc]));
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}


// ---------------------------------------------------------------- CTA-pair GEMM
// The same GEMM on 256 x 256 output tiles, each computed by a cluster of two CTAs on the
// two SMs of a TPC with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16). Each CTA
// holds, per stage, its 128 rows of A and its 128 rows (output columns) of B -- 32 KB, so
// six stages -- and its 128 output rows of the accumulator in its own tensor memory. One
// MMA reads both CTAs' tiles, so each SM's shared memory supplies half of B instead of
// all of it: the operand traffic per SM per K-step drops from 12 KB to 8 KB, which is
// what bounds the one-CTA kernel.
//   - producer (warp 0 of each CTA): waits for its stage's release, loads its A and B
//     tiles by TMA; the bytes of both CTAs are counted on the leader's full barrier, which
//     the leader's producer arms for 64 KB;
//   - MMA (warp 1 of the leader): waits on full, issues 4 MMAs per stage, and releases the
//     stage in both CTAs with one multicast commit; after a tile, a multicast commit marks
//     the accumulator full in both CTAs;
//   - epilogue (warps 2..5 of each CTA): its 128 rows from its own tensor memory, then an
//     arrival on the leader's accumulator-empty barrier (8 arrivals: 4 warps x 2 CTAs).
// Teardown: each producer waits until every stage it loaded was released (no multicast
// arrival can reach an exited CTA), the leader's MMA warp waits until both CTAs'
// epilogues released both accumulators, then the two MMA warps hand a token to each other
// through mbarriers (bounded waits) before both deallocate the pair's tensor memory.
constexpr int PB_M = 256, PB_N = 256;  // the pair's tile
constexpr int PA_BYTES = 128 * BK * 2, PB_BYTES = 128 * BK * 2;
constexpr int P_STAGE_BYTES = PA_BYTES + PB_BYTES;  // 32 KB per CTA
constexpr int P_STAGES = 6;
constexpr uint32_t P_IDESC = idesc_bf16_f32(PB_M, PB_N, false, false);
constexpr size_t P_SMEM_BYTES = 1024 + P_STAGES * P_STAGE_BYTES + 256;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_bf16_tn_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                             Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = base + P_STAGES * PA_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + P_STAGES * P_STAGE_BYTES);
  uint64_t* full = bars;                          // [P_STAGES] (the leader's is used)
  uint64_t* empty = bars + P_STAGES;              // [P_STAGES]
  uint64_t* tfull = bars + 2 * P_STAGES;          // [NUM_ACC]
  uint64_t* tempty = bars + 2 * P_STAGES + NUM_ACC;  // [NUM_ACC] (the leader's is used)
  uint64_t* token = bars + 2 * P_STAGES + 2 * NUM_ACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(token + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1), pairs = static_cast<int>(gridDim.x >> 1);
  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), 1);
    }
    for (int a = 0; a < NUM_ACC; ++a) {
      mbar_init(smem_addr(&tfull[a]), 1);
      mbar_init(smem_addr(&tempty[a]), 8);
    }
    mbar_init(smem_addr(token), 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_addr(tmem_slot), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before either CTA arrives on the other's
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = p.tiles_m * p.tiles_n;
  const uint32_t full_at_leader = mapa_shared(smem_addr(&full[0]), 0);
  const uint32_t tempty_at_leader = mapa_shared(smem_addr(&tempty[0]), 0);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += pairs) {
        int tm, tn;
        tile_coords(p, tile, tm, tn);
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait_site(smem_addr(&empty[stage]), phase ^ 1, 26, kb)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(smem_addr(&full[stage]), 2 * P_STAGE_BYTES);
          const uint32_t bar = full_at_leader + 8 * stage;
          tma_load_2d_pair(smem_addr(sA + stage * PA_BYTES), &tmap_a, bar, kb * BK, tm * PB_M + 128 * rank);
          tma_load_2d_pair(smem_addr(sB + stage * PB_BYTES), &tmap_b, bar, kb * BK, tn * PB_N + 128 * rank);
          if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // every stage this CTA loaded has been released by the pair's MMAs
      for (int s = 0; s < P_STAGES; ++s) {
        if (!mbar_wait_site(smem_addr(&empty[stage]), phase ^ 1, 27, s)) break;
        if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    int it = 0;
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += pairs, ++it) {
        const int acc = it & 1;
        if (!mbar_wait_site(smem_addr(&tempty[acc]), ((it >> 1) & 1) ^ 1, 28, it)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * PB_N;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait_site(smem_addr(&full[stage]), phase, 29, kb)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_addr(sA + stage * PA_BYTES), b0 = smem_addr(sB + stage * PB_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            tc_mma_f16_pair(d_tmem, sw128_kmajor_desc(a0 + kk * 32), sw128_kmajor_desc(b0 + kk * 32), P_IDESC,
                            (kb | kk) != 0);
          tc_commit_pair(smem_addr(&empty[stage]), 0x3);
          if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
        }
        tc_commit_pair(smem_addr(&tfull[acc]), 0x3);
      }
      // both CTAs' epilogues have released both accumulators (the last uses of each)
      for (int a = 0; a < NUM_ACC && it > a; ++a) {
        const int last = it - 1 - ((it - 1 - a) & 1);  // the last tile that used accumulator (it - 1 - a) & 1
        mbar_wait_site(smem_addr(&tempty[last & 1]), (last >> 1) & 1, 30, last);
      }
    }
    __syncwarp();
  } else {
    const int quarter = warp & 3;
    int it = 0;
    for (int tile = pair; tile < num_tiles; tile += pairs, ++it) {
      const int acc = it & 1;
      if (!mbar_wait_warp(smem_addr(&tfull[acc]), (it >> 1) & 1, 31, it)) break;
      tc_fence_after();
      int tm, tn;
      tile_coords(p, tile, tm, tn);
      const int row = tm * PB_M + 128 * static_cast<int>(rank) + quarter * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * PB_N;
#pragma unroll 1
      for (int c = 0; c < PB_N; c += 32) {
        uint32_t r[32];
        tmem_ld32(taddr + c, r);
        tc_wait_ld();
        reg_fence32(r);
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        store_row32(p, row, tn * PB_N + c, v);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_at_leader + 8 * acc);
    }
  }
  __syncthreads();
  if (warp == 1) {
    // the peer tells the leader it is done, the leader answers: after this neither CTA's
    // tensor memory or shared memory is used by the other
    if (lane == 0) {
      if (!leader) {
        mbar_arrive_cluster(mapa_shared(smem_addr(token), 0));
        mbar_wait_site(smem_addr(token), 0, 32, 0);
      } else {
        mbar_wait_site(smem_addr(token), 0, 32, 0);
        mbar_arrive_cluster(mapa_shared(smem_addr(token), 1));
      }
    }
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace gemm
}  // namespace faq

using namespace faq;

namespace faq {
namespace gemm {
// The SM count the persistent GEMMs (K3, K3p) size their grids for; 0: every SM. A
// tensor-parallel caller lowers it while collectives run beside its GEMMs, so that the
// collective kernels find free SMs instead of waiting for a GEMM that holds all of them.
static std::atomic<int> g_sm_target{0};
static int grid_sms() {
  const int all = num_sms(), t = g_sm_target.load(std::memory_order_relaxed);
  return t > 0 && t < all ? std::max(2, t) : all;
}
// FAQ_GEMM_ONE_SM=1 in the environment keeps every GEMM on the one-CTA kernel
static bool one_sm_forced() {
  static const bool forced = [] {
    const char* e = std::getenv("FAQ_GEMM_ONE_SM");
    return e != nullptr && e[0] == '1';
  }();
  return forced;
}
}  // namespace gemm
}  // namespace faq

extern "C" int faq_gemm_bf16_tn_residual(const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m,
                                         int64_t n, int64_t k, const void* bias, const void* residual, int64_t ldr,
                                         void* y, int64_t ldy, void* stream) {
  FAQ_CHECK_ARG(a && b && y, "null pointer");
  FAQ_CHECK_ARG(residual == nullptr || ldr >= n, "residual leading dimension too small");
  FAQ_CHECK_ARG(m >= 0 && n >= 0 && k > 0, "bad shape");
  FAQ_CHECK_ARG(m < (int64_t(1) << 31) && n < (int64_t(1) << 31) && k < (int64_t(1) << 31), "shape too large");
  FAQ_CHECK_ARG(lda >= k && ldb >= k && ldy >= n, "leading dimension too small");
  FAQ_CHECK_ARG(lda % 8 == 0 && ldb % 8 == 0 && k % 8 == 0, "TMA needs lda, ldb and k multiples of 8");
  FAQ_CHECK_ARG(aligned16(a) && aligned16(b), "a and b must be 16-byte aligned");
  if (m == 0 || n == 0) return FAQ_OK;
  using namespace faq::gemm;
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
    const uint64_t strides[1] = {static_cast<uint64_t>(lda) * 2};
    const uint32_t box[2] = {BK, BM};
    int rc = make_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != FAQ_OK) return rc;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(n)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldb) * 2};
    const uint32_t box[2] = {BK, BN};
    int rc = make_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != FAQ_OK) return rc;
  }
  Params p;
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.kblocks = static_cast<int>((k + BK - 1) / BK);
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.ldr = ldr;
  p.r_vec = residual != nullptr && aligned16(residual) && ldr % 8 == 0;
  p.y = static_cast<__nv_bfloat16*>(y);
  p.ldy = ldy;
  p.y_vec = aligned16(y) && ldy % 8 == 0;
  if (m >= PB_M && n >= PB_N && !one_sm_forced()) {
    // CTA pairs on 256 x 256 tiles: A as 128-row boxes (each CTA its half), B likewise
    CUtensorMap tb2;
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(n)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldb) * 2};
    const uint32_t box[2] = {BK, 128};
    int rc = make_tmap(&tb2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != FAQ_OK) return rc;
    p.tiles_m = static_cast<int>((m + PB_M - 1) / PB_M);
    p.tiles_n = static_cast<int>((n + PB_N - 1) / PB_N);
    p.group_m = std::max(1, std::min(p.tiles_m, 8));  // 8 pair rows = 2048 rows of A per group
    const int tiles = p.tiles_m * p.tiles_n;
    const int grid = 2 * std::max(1, std::min(tiles, grid_sms() / 2));
    FAQ_CUDA(cudaFuncSetAttribute(gemm_bf16_tn_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(P_SMEM_BYTES)));
    gemm_bf16_tn_pair_kernel<<<grid, THREADS, P_SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(ta, tb2, p);
    return launch_status("gemm_bf16_tn_pair_kernel");
  }
  p.tiles_m = static_cast<int>((m + BM - 1) / BM);
  p.tiles_n = static_cast<int>((n + BN - 1) / BN);
  // about sqrt(148 * B panel / A panel) = sqrt(148 * 2) ~ 17 M tiles per group minimizes
  // the panels a wave reads (G A panels + 148 / G B panels, B panels twice as large)
  p.group_m = std::max(1, std::min(p.tiles_m, 16));
  const int tiles = p.tiles_m * p.tiles_n;
  const int grid = std::min(tiles, grid_sms());
  FAQ_CUDA(cudaFuncSetAttribute(gemm_bf16_tn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(SMEM_BYTES)));
  gemm_bf16_tn_kernel<<<grid, THREADS, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(ta, tb, p);
  return launch_status("gemm_bf16_tn_kernel");
}

extern "C" int faq_set_gemm_sm_target(int sms) {
  FAQ_CHECK_ARG(sms >= 0, "sms must be >= 0 (0: every SM)");
  faq::gemm::g_sm_target.store(sms, std::memory_order_relaxed);
  return FAQ_OK;
}

extern "C" int faq_gemm_bf16_tn(const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m, int64_t n,
                                int64_t k, const void* bias, void* y, int64_t ldy, void* stream) {
  return faq_gemm_bf16_tn_residual(a, lda, b, ldb, m, n, k, bias, nullptr, 0, y, ldy, stream);
}
