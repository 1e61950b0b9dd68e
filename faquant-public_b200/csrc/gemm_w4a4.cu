// K3p -- W4A4 GEMM on packed HiF4 operands: y = deq(A) . deq(B)^T (+ bias) (+ residual).
//
// The operands stay in the 4.5-bit packed format of include/faquant_b200.h in HBM (codes
// uint8 [rows, k/2], one uint32 meta word per 64 values) and are expanded tile by tile
// into the 128-byte-swizzled bf16 shared-memory layout the tensor cores read, so HBM and
// L2 carry 0.5625 bytes per operand value instead of 2. Every HiF4 value is exact in
// bf16 and the MMA sequence is the one of the bf16 GEMM (gemm_sm100.cu: the same 64-wide
// K blocks, the same four K=16 MMAs per block, the same order), so the output is
// bit-identical to faq_gemm_bf16_tn on the dequantized operands -- the reference's
// F.linear on its fake-quantized tensors (quantization.py:277, hif4.py:254-271).
//
// CTA pairs (cluster of two, tcgen05.mma.cta_group::2, 256 x 256 output tiles, persistent):
//   warp 0        producer: TMA of this CTA's packed rows of each K block -- codes as a
//                 [128 rows x 32 B] box, meta as a [128 x 16 B] box (the aligned group of
//                 four blocks holding this one) -- into a staging ring (sizes: Rings);
//   warp 1        TMEM allocation; the leader's lane 0 issues the MMAs and commits;
//   warps 2..5    epilogue, as in the bf16 pair kernel;
//   warps 6..13   transform: thread t owns row t/2 of this CTA's 128 rows and half t%2 of
//                 the 64-value block; it reads its 16 code bytes and the meta word of each
//                 operand from the staging slot, expands them and
//                 stores four 16-byte chunks into the swizzled bf16 tile of the operand
//                 ring; then fence.proxy.async and one arrival per warp at CTA scope: in
//                 the leader on the MMA's full barrier, in the peer on a local barrier;
//                 and on the slot's empty barrier;
//   warp 14       the peer's forwarder: one arrival per stage on the leader's full barrier,
//                 release at cluster scope (the MMA issuer acquires at cluster scope);
//   warp 15       when A is given as K1's bf16 QDQ output: TMA of the bf16 A tile into the
//                 operand ring (its own warp, so the staging ring never waits behind it). The packed bytes come by TMA, not by loads of these threads,
//                 because a release must first complete every earlier load of the
//                 releasing thread: loads issued ahead would each cost a full memory
//                 round trip per K block.
// Expansion of one 32-bit code word (8 values, sign-magnitude nibbles s|m, value =
// (-1)^s (m/4) scale 2^(lv2+lv3)): r = the word rotated left by 4, so that byte j of r
// carries nibble 2j's sign in bit 7 and nibble 2j+1 in bits 0..3; one byte permute per
// pair of values gathers [m0 | s0<<15 | m1<<16 | s1<<31] (plus junk bits); the bf16 pair
// (128 + m0, 128 + m1) = (x & 0x00070007) | 0x43004300 is exact (bf16 spacing 1 on
// [128, 256)); one bf16x2 FMA with (c, -128 c), c = scale 2^(lv2+lv3-2) a power-of-two
// shift of the E6M2 scale, gives m c exactly (at most 6 significant bits, a single
// rounding of an exact result); xor with the gathered sign bits restores the sign, -0.0
// for a negative zero code as the packed format's own decoder gives. Four integer ops
// and one FMA per pair, plus the scale words per 4-value lv3 group.
#include "common.cuh"
#include "hif4.cuh"
#include "tma.h"

namespace faq {
namespace w4a4 {

constexpr int BK = 64;  // one HiF4 block of K per stage
constexpr int TILE_BYTES = 128 * BK * 2;     // one CTA's 128 rows of one operand, bf16
constexpr int STAGE_BYTES = 2 * TILE_BYTES;  // A half + B half
constexpr int KB_PER_ROUND = 2;  // K blocks a transform warp expands between two fences
constexpr uint32_t kSuspendNs = 0;  // suspend hint of the polling warps' waits
// packed staging slot: per operand 128 rows x 32 code bytes, then 128 rows x 16 meta bytes
constexpr int P_CODES = 128 * 32;
constexpr int P_META = 128 * 16;
constexpr int P_OPERAND = P_CODES + P_META;

constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = 512;
constexpr int TRANSFORM_WARPS = 8;
// Warp roles. A warp runs on sub-partition (SMSP) warp % 4. The MMA issuer is a single
// thread whose few instructions per K block must not wait behind the integer-heavy
// expansion, so its sub-partition (1) holds no transform warp: only the issuer, one
// epilogue warp and the two single-lane roles. The eight transform warps share the other
// three sub-partitions (3, 3, 2).
constexpr int PRODUCER_WARP = 0, MMA_WARP = 1, FORWARD_WARP = 9, A_WARP = 13;
constexpr int FIRST_EPILOGUE_WARP = 4;  // warps 4..7: TMEM lane quarter = warp % 4
constexpr int THREADS = 16 * 32;        // 512
// transform warp index (0..7) of each warp, -1 for the other roles
__device__ __forceinline__ int transform_index(int warp) {
  // warps 2, 3, 8, 10, 11, 12, 14, 15
  constexpr unsigned long long kMap = 0x76F543F2FFFF10FFull;  // nibble w: index or F
  const int v = static_cast<int>((kMap >> (4 * warp)) & 0xF);
  return v == 0xF ? -1 : v;
}
constexpr int DRAINER_WARP = 2;  // transform index 0
constexpr uint32_t IDESC = idesc_bf16_f32(256, 256, false, false);
// Ring sizes per mode. Both operands packed: 4 operand stages and 8 staging slots of A and
// B (12 KB). Activation as bf16 by TMA, only the weight staged: 6 operand stages and 4
// slots of B (6 KB) -- the operand ring then also covers the TMA latency of the A tiles.
template <bool A_PACKED>
struct Rings {
  static constexpr int STAGES = A_PACKED ? 4 : 6;
  static constexpr int PSTAGES = A_PACKED ? 8 : 4;
  static constexpr int P_SLOT = A_PACKED ? 2 * P_OPERAND : P_OPERAND;  // [A,] B
  static constexpr int P_B = A_PACKED ? P_OPERAND : 0;                 // B's offset in a slot
  static constexpr int NUM_BARS = 3 * STAGES + 2 * PSTAGES + 2 * NUM_ACC + 1;
  static constexpr size_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + PSTAGES * P_SLOT + NUM_BARS * 8 + 16;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory of the packed GEMM");
  static_assert(STAGES % KB_PER_ROUND == 0 && PSTAGES % KB_PER_ROUND == 0, "rounds tile the rings");
};

struct Params {
  gemm::Params g;  // shape, tile order and epilogue (bias, residual, output)
};

// One operand's share of one K block for this thread: 32 values (16 code bytes) and the
// block's meta word.
struct Slice {
  uint4 codes;
  uint32_t meta;
};

__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
// This thread's slice of an operand from a staging slot (`operand` = its shared address).
__device__ __forceinline__ Slice read_slice(uint32_t operand, int row, int half, int kb) {
  Slice s;
  s.codes = lds_v4(operand + static_cast<uint32_t>(row * 32 + half * 16));
  s.meta = lds_u32(operand + P_CODES + static_cast<uint32_t>(row * 16 + (kb & 3) * 4));
  return s;
}
__device__ __forceinline__ void sts_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// Expand one thread's 32 values (half `half` of a 64-value block) into row `row` of a
// 128-byte-swizzled K-major bf16 tile at `tile` (shared address, 1024-byte aligned).
__device__ __forceinline__ void expand_half(const Slice& s, int half, uint32_t tile, int row) {
  uint32_t out[16];
  hif4_expand32_bf16(s.codes, s.meta, half, out);  // hif4.cuh: three ALU ops and one bf16x2 FMA per pair
  const uint32_t row_addr = tile + static_cast<uint32_t>(row) * 128u;
  const uint32_t swz = static_cast<uint32_t>(row & 7);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t chunk = static_cast<uint32_t>(4 * half + i) ^ swz;
    sts_v4(row_addr + (chunk << 4), out[4 * i], out[4 * i + 1], out[4 * i + 2], out[4 * i + 3]);
  }
}

// The packed operand maps of one GEMM (codes 2-D uint8 [rows, k/2], box 32 x 128; meta 2-D
// uint32 [rows, k/64], box 4 x 128) and the bf16 A map when A comes as K1's QDQ output.
struct Maps {
  CUtensorMap a_bf16, a_codes, a_meta, b_codes, b_meta;
};

template <bool A_PACKED>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    w4a4_gemm_pair_kernel(const __grid_constant__ Maps maps, const __grid_constant__ Params p) {
  constexpr int STAGES = Rings<A_PACKED>::STAGES, PSTAGES = Rings<A_PACKED>::PSTAGES;
  constexpr int P_SLOT = Rings<A_PACKED>::P_SLOT, P_B = Rings<A_PACKED>::P_B;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = base + STAGES * TILE_BYTES;
  uint8_t* sP = base + STAGES * STAGE_BYTES;  // packed staging slots
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + PSTAGES * P_SLOT);
  uint64_t* full = bars;                                   // [STAGES] (the leader's is used)
  uint64_t* empty = bars + STAGES;                         // [STAGES]
  uint64_t* pfull = bars + 2 * STAGES;                     // [PSTAGES] staging slot loaded
  uint64_t* pempty = bars + 2 * STAGES + PSTAGES;          // [PSTAGES] staging slot read
  uint64_t* tfull = bars + 2 * STAGES + 2 * PSTAGES;       // [NUM_ACC]
  uint64_t* tempty = tfull + NUM_ACC;                      // [NUM_ACC] (the leader's is used)
  uint64_t* token = tempty + NUM_ACC;
  uint64_t* ready = token + 1;                             // [STAGES] the peer's transform warps done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ready + STAGES);
  const gemm::Params& g = p.g;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1), pairs = static_cast<int>(gridDim.x >> 1);
  if (threadIdx.x == 0) {
    // full (the leader's): one arrival per leader transform warp, one from the peer's
    // forwarder, plus the leader producer's arrive.expect_tx when A comes by TMA;
    // ready (the peer's): one arrival per peer transform warp
    const uint32_t full_count = TRANSFORM_WARPS + 1 + (A_PACKED ? 0 : 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_addr(&full[s]), full_count);
      mbar_init(smem_addr(&empty[s]), 1);
      mbar_init(smem_addr(&ready[s]), TRANSFORM_WARPS);
    }
    for (int s = 0; s < PSTAGES; ++s) {
      mbar_init(smem_addr(&pfull[s]), 1);
      mbar_init(smem_addr(&pempty[s]), TRANSFORM_WARPS);
    }
    for (int a = 0; a < NUM_ACC; ++a) {
      mbar_init(smem_addr(&tfull[a]), 1);
      mbar_init(smem_addr(&tempty[a]), 8);
    }
    mbar_init(smem_addr(token), 1);
    fence_barrier_init();
    if constexpr (!A_PACKED) tma_prefetch_desc(&maps.a_bf16);
    if constexpr (A_PACKED) {
      tma_prefetch_desc(&maps.a_codes);
      tma_prefetch_desc(&maps.a_meta);
    }
    tma_prefetch_desc(&maps.b_codes);
    tma_prefetch_desc(&maps.b_meta);
  }
  if (warp == MMA_WARP) {
    tmem_alloc_pair(smem_addr(tmem_slot), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before either CTA arrives on the other's
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = g.tiles_m * g.tiles_n;
  const uint32_t full_at_leader = mapa_shared(smem_addr(&full[0]), 0);
  const uint32_t tempty_at_leader = mapa_shared(smem_addr(&tempty[0]), 0);
  const int my_rows = 128 * static_cast<int>(rank);

  const int tw = transform_index(warp);
  if (warp == PRODUCER_WARP) {
    if (lane == 0) {
      int ps = 0;
      uint32_t pphase = 0;
      bool ok = true;
      constexpr uint32_t slot_bytes = P_SLOT;
      for (int tile = pair; tile < num_tiles && ok; tile += pairs) {
        int tm, tn;
        gemm::tile_coords(g, tile, tm, tn);
        for (int kb = 0; kb < g.kblocks; ++kb) {
          if (!mbar_wait_site(smem_addr(&pempty[ps]), pphase ^ 1, 60, kb)) { ok = false; break; }
          const uint32_t pbar = smem_addr(&pfull[ps]);
          const uint32_t slot = smem_addr(sP + ps * P_SLOT);
          mbar_arrive_expect_tx(pbar, slot_bytes);
          if constexpr (A_PACKED) {
            tma_load_2d(slot, &maps.a_codes, pbar, kb * 32, tm * 256 + my_rows);
            tma_load_2d(slot + P_CODES, &maps.a_meta, pbar, kb & ~3, tm * 256 + my_rows);
          }
          tma_load_2d(slot + P_B, &maps.b_codes, pbar, kb * 32, tn * 256 + my_rows);
          tma_load_2d(slot + P_B + P_CODES, &maps.b_meta, pbar, kb & ~3, tn * 256 + my_rows);
          if (++ps == PSTAGES) { ps = 0; pphase ^= 1; }
        }
      }
      // the staging loads landed (the transform warps read every slot)
      for (int s = 0; s < PSTAGES; ++s) {
        if (!mbar_wait_site(smem_addr(&pempty[ps]), pphase ^ 1, 69, s)) break;
        if (++ps == PSTAGES) { ps = 0; pphase ^= 1; }
      }
    }
    __syncwarp();
  } else if (warp == A_WARP) {
    // bf16 A (K1's QDQ output) by TMA into the operand ring, on its own warp so that the
    // staging loads above never wait behind the operand ring's releases
    if constexpr (!A_PACKED) {
      if (lane == 0) {
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int tile = pair; tile < num_tiles && ok; tile += pairs) {
          int tm, tn;
          gemm::tile_coords(g, tile, tm, tn);
          for (int kb = 0; kb < g.kblocks; ++kb) {
            if (!mbar_wait_site(smem_addr(&empty[stage]), phase ^ 1, 61, kb)) { ok = false; break; }
            if (leader) mbar_arrive_expect_tx(smem_addr(&full[stage]), 2 * TILE_BYTES);
            tma_load_2d_pair(smem_addr(sA + stage * TILE_BYTES), &maps.a_bf16, full_at_leader + 8 * stage,
                             kb * BK, tm * 256 + my_rows);
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
        }
        // every operand stage this CTA loaded was released by the pair's MMAs
        for (int s = 0; s < STAGES; ++s) {
          if (!mbar_wait_site(smem_addr(&empty[stage]), phase ^ 1, 70, s)) break;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    int it = 0;
    const uint32_t desc_a0 = sw128_desc_lo(smem_addr(sA), 16), desc_b0 = sw128_desc_lo(smem_addr(sB), 16);
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += pairs, ++it) {
        const int acc = it & 1;
        if (!mbar_wait_site(smem_addr(&tempty[acc]), ((it >> 1) & 1) ^ 1, 62, it)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * 256;
        for (int kb = 0; kb < g.kblocks; ++kb) {
          // transform warps of the peer CTA released their stores at cluster scope
          if (!mbar_wait_cluster_site(smem_addr(&full[stage]), phase, 63, kb)) { ok = false; break; }
          tc_fence_after();
          // descriptor low words (start address >> 4 | leading byte offset 16 >> 4 << 16);
          // a K=16 step advances the start by 32 bytes
          const uint32_t a_lo = desc_a0 + static_cast<uint32_t>(stage) * (TILE_BYTES >> 4);
          const uint32_t b_lo = desc_b0 + static_cast<uint32_t>(stage) * (TILE_BYTES >> 4);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            tc_mma_f16_pair_lo(d_tmem, a_lo + 2 * kk, b_lo + 2 * kk, IDESC, (kb | kk) != 0);
          tc_commit_pair(smem_addr(&empty[stage]), 0x3);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        tc_commit_pair(smem_addr(&tfull[acc]), 0x3);
      }
      for (int a = 0; a < NUM_ACC && it > a; ++a) {
        const int last = it - 1 - ((it - 1 - a) & 1);
        mbar_wait_site(smem_addr(&tempty[last & 1]), (last >> 1) & 1, 64, last);
      }
    }
    __syncwarp();
  } else if (warp == FORWARD_WARP) {
    // The peer CTA's transform warps arrive at CTA scope on `ready`; this lane forwards each
    // completed stage to the leader's full barrier with one release at cluster scope. A
    // cluster-scope release costs about a thousand cycles (the CTA's stores must become
    // visible to the pair), so it is paid once per stage here, off the transform warps'
    // path, instead of once per transform warp.
    if (!leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      const int items = ((num_tiles - pair + pairs - 1) / pairs) * g.kblocks;
      for (int i = 0; i < items; ++i) {
        if (!mbar_wait_site(smem_addr(&ready[stage]), phase, 72, i)) break;
        mbar_arrive_cluster(full_at_leader + 8 * stage);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    __syncwarp();
  } else if (tw < 0) {  // epilogue warps 4..7
    const int quarter = warp & 3;
    int it = 0;
    for (int tile = pair; tile < num_tiles; tile += pairs, ++it) {
      const int acc = it & 1;
      if (!mbar_wait_warp_suspend(smem_addr(&tfull[acc]), (it >> 1) & 1, kSuspendNs, 65, it)) break;
      tc_fence_after();
      int tm, tn;
      gemm::tile_coords(g, tile, tm, tn);
      const int row = tm * 256 + 128 * static_cast<int>(rank) + quarter * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * 256;
#pragma unroll 1
      for (int c = 0; c < 256; c += 32) {
        uint32_t r[32];
        tmem_ld32(taddr + c, r);
        tc_wait_ld();
        reg_fence32(r);
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        gemm::store_row32(g, row, tn * 256 + c, v);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_at_leader + 8 * acc);
    }
  } else {
    // transform warps
    const int t = tw * 32 + lane;
    const int row = t >> 1, half = t & 1;
    const bool drainer = warp == DRAINER_WARP;
    int stage = 0, ps = 0, n = 0;
    uint32_t phase = 0, pphase = 0;
    bool ok = true;
    // Two K blocks per round: one fence and one set of arrivals serve both (the proxy fence
    // and the cluster-scope release are the costly steps of a round). kblocks is a
    // multiple of 4 (k % 256 == 0), so a round never straddles two tiles.
    for (int tile = pair; tile < num_tiles && ok; tile += pairs) {
      for (int kb = 0; kb < g.kblocks; kb += KB_PER_ROUND, n += KB_PER_ROUND) {
        Slice sa[KB_PER_ROUND] = {}, sb[KB_PER_ROUND];
#pragma unroll
        for (int r = 0; r < KB_PER_ROUND; ++r) {
          const int q = (ps + r) % PSTAGES;
          const uint32_t qphase = pphase ^ static_cast<uint32_t>(ps + r >= PSTAGES);
          if (!mbar_wait_warp_suspend(smem_addr(&pfull[q]), qphase, kSuspendNs, 66, n + r)) ok = false;
          const uint32_t slot = smem_addr(sP + q * P_SLOT);
          if constexpr (A_PACKED) sa[r] = read_slice(slot, row, half, kb + r);
          sb[r] = read_slice(slot + P_B, row, half, kb + r);
        }
        if (!ok) break;
        {
          // Free the staging slots as soon as every lane holds its values: the xor below
          // depends on every loaded register, so a lane reaches the __syncwarp only once
          // its loads from the slots have completed (a load still in flight could be
          // overwritten by the next TMA into the slot).
          uint32_t dep = 0;
#pragma unroll
          for (int r = 0; r < KB_PER_ROUND; ++r) {
            dep ^= sb[r].codes.x ^ sb[r].codes.y ^ sb[r].codes.z ^ sb[r].codes.w ^ sb[r].meta;
            if constexpr (A_PACKED) dep ^= sa[r].codes.x ^ sa[r].codes.y ^ sa[r].codes.z ^ sa[r].codes.w ^ sa[r].meta;
          }
          asm volatile("" ::"r"(dep));
          __syncwarp();
          if (lane == 0) {
#pragma unroll
            for (int r = 0; r < KB_PER_ROUND; ++r) mbar_arrive(smem_addr(&pempty[(ps + r) % PSTAGES]));
          }
        }
#pragma unroll
        for (int r = 0; r < KB_PER_ROUND; ++r) {
          const int st = (stage + r) % STAGES;
          const uint32_t sphase = phase ^ static_cast<uint32_t>(stage + r >= STAGES);
          if (!mbar_wait_warp_suspend(smem_addr(&empty[st]), sphase ^ 1, kSuspendNs, 67, n + r)) { ok = false; break; }
          if constexpr (A_PACKED) expand_half(sa[r], half, smem_addr(sA + st * TILE_BYTES), row);
          expand_half(sb[r], half, smem_addr(sB + st * TILE_BYTES), row);
        }
        if (!ok) break;
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
#pragma unroll
          for (int r = 0; r < KB_PER_ROUND; ++r) {
            const int st = (stage + r) % STAGES;
            mbar_arrive(smem_addr(leader ? &full[st] : &ready[st]));
          }
        }
        ps += KB_PER_ROUND;
        if (ps >= PSTAGES) { ps -= PSTAGES; pphase ^= 1; }
        stage += KB_PER_ROUND;
        if (stage >= STAGES) { stage -= STAGES; phase ^= 1; }
      }
    }
    // every operand stage this CTA filled has been released by the pair's MMAs: no commit
    // can arrive at this CTA's barriers after it exits
    if (drainer) {
      for (int s = 0; s < STAGES; ++s) {
        if (!mbar_wait_warp(smem_addr(&empty[stage]), phase ^ 1, 68, s)) break;
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  }
  __syncthreads();
  if (warp == MMA_WARP) {
    if (lane == 0) {
      if (!leader) {
        mbar_arrive_cluster(mapa_shared(smem_addr(token), 0));
        mbar_wait_site(smem_addr(token), 0, 71, 0);
      } else {
        mbar_wait_site(smem_addr(token), 0, 71, 0);
        mbar_arrive_cluster(mapa_shared(smem_addr(token), 1));
      }
    }
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

static int launch(Maps& maps, bool a_packed, Params& p, void* stream) {
  gemm::Params& g = p.g;
  g.tiles_m = (g.m + 255) / 256;
  g.tiles_n = (g.n + 255) / 256;
  g.kblocks = g.k / BK;
  g.group_m = std::max(1, std::min(g.tiles_m, 8));
  const int tiles = g.tiles_m * g.tiles_n;
  const int grid = 2 * std::max(1, std::min(tiles, faq::gemm::grid_sms() / 2));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a_packed) {
    constexpr size_t smem = Rings<true>::SMEM_BYTES;
    FAQ_CUDA(cudaFuncSetAttribute(w4a4_gemm_pair_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(smem)));
    w4a4_gemm_pair_kernel<true><<<grid, THREADS, smem, s>>>(maps, p);
    return launch_status("w4a4_gemm_pair_kernel<packed A>");
  }
  constexpr size_t smem = Rings<false>::SMEM_BYTES;
  FAQ_CUDA(cudaFuncSetAttribute(w4a4_gemm_pair_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem)));
  w4a4_gemm_pair_kernel<false><<<grid, THREADS, smem, s>>>(maps, p);
  return launch_status("w4a4_gemm_pair_kernel<bf16 A>");
}

// Tensor maps of one packed operand of `rows` rows: codes box 32 B x 128 rows, meta box
// 4 words x 128 rows (rows beyond `rows` read as zeros).
static int packed_maps(const uint8_t* codes, const uint32_t* meta, int64_t rows, int64_t k, const char* what,
                       CUtensorMap* mc, CUtensorMap* mm) {
  FAQ_CHECK_ARG(codes != nullptr && meta != nullptr, std::string(what) + ": null codes or meta");
  FAQ_CHECK_ARG(aligned16(codes) && aligned16(meta), std::string(what) + ": codes and meta must be 16-byte aligned");
  const uint64_t cd[2] = {static_cast<uint64_t>(k / 2), static_cast<uint64_t>(rows)};
  const uint64_t cs[1] = {static_cast<uint64_t>(k / 2)};
  const uint32_t cb[2] = {32, 128};
  int rc = make_tmap(mc, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, codes, cd, cs, cb, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc != FAQ_OK) return rc;
  const uint64_t md[2] = {static_cast<uint64_t>(k / 64), static_cast<uint64_t>(rows)};
  const uint64_t ms[1] = {static_cast<uint64_t>(k / 64) * 4};
  const uint32_t mb[2] = {4, 128};
  return make_tmap(mm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, meta, md, ms, mb, CU_TENSOR_MAP_SWIZZLE_NONE);
}

static int setup(Params& p, Maps& maps, int64_t m, int64_t n, int64_t k, const uint8_t* b_codes,
                 const uint32_t* b_meta, const void* bias, const void* residual, int64_t ldr, void* y, int64_t ldy) {
  FAQ_CHECK_ARG(y != nullptr, "null output");
  FAQ_CHECK_ARG(m >= 0 && n >= 0 && k > 0, "bad shape");
  FAQ_CHECK_ARG(k % 64 == 0, "k must be a multiple of 64 (whole HiF4 blocks)");
  FAQ_CHECK_ARG(m < (int64_t(1) << 31) && n < (int64_t(1) << 31) && k < (int64_t(1) << 31), "shape too large");
  FAQ_CHECK_ARG(ldy >= n, "output leading dimension too small");
  FAQ_CHECK_ARG(residual == nullptr || ldr >= n, "residual leading dimension too small");
  if (k % 256 != 0)
    return fail(FAQ_ERR_UNSUPPORTED, "the packed GEMM loads meta rows by TMA: k must be a multiple of 256 "
                                     "(16-byte meta rows); use faq_gemm_bf16_tn on the dequantized operands");
  std::memset(&maps, 0, sizeof(maps));
  if (n > 0) {
    int rc = packed_maps(b_codes, b_meta, n, k, "b", &maps.b_codes, &maps.b_meta);
    if (rc) return rc;
  }
  gemm::Params& g = p.g;
  g.m = static_cast<int>(m);
  g.n = static_cast<int>(n);
  g.k = static_cast<int>(k);
  g.bias = static_cast<const __nv_bfloat16*>(bias);
  g.residual = static_cast<const __nv_bfloat16*>(residual);
  g.ldr = ldr;
  g.r_vec = residual != nullptr && aligned16(residual) && ldr % 8 == 0;
  g.y = static_cast<__nv_bfloat16*>(y);
  g.ldy = ldy;
  g.y_vec = aligned16(y) && ldy % 8 == 0;
  return FAQ_OK;
}

}  // namespace w4a4
}  // namespace faq

extern "C" int faq_w4a4_gemm(const uint8_t* a_codes, const uint32_t* a_meta, const uint8_t* b_codes,
                             const uint32_t* b_meta, int64_t m, int64_t n, int64_t k, const void* bias,
                             const void* residual, int64_t ldr, void* y, int64_t ldy, void* stream) {
  using namespace faq;
  w4a4::Params p;
  w4a4::Maps maps;
  int rc = w4a4::setup(p, maps, m, n, k, b_codes, b_meta, bias, residual, ldr, y, ldy);
  if (rc) return rc;
  if (m == 0 || n == 0) return FAQ_OK;
  rc = w4a4::packed_maps(a_codes, a_meta, m, k, "a", &maps.a_codes, &maps.a_meta);
  if (rc) return rc;
  return w4a4::launch(maps, true, p, stream);
}

extern "C" int faq_w4a4_gemm_qdq_a(const void* a, int64_t lda, const uint8_t* b_codes, const uint32_t* b_meta,
                                   int64_t m, int64_t n, int64_t k, const void* bias, const void* residual,
                                   int64_t ldr, void* y, int64_t ldy, void* stream) {
  using namespace faq;
  w4a4::Params p;
  w4a4::Maps maps;
  int rc = w4a4::setup(p, maps, m, n, k, b_codes, b_meta, bias, residual, ldr, y, ldy);
  if (rc) return rc;
  FAQ_CHECK_ARG(a != nullptr && aligned16(a), "a must be a 16-byte aligned device pointer");
  FAQ_CHECK_ARG(lda >= k && lda % 8 == 0, "lda must be >= k and a multiple of 8");
  if (m == 0 || n == 0) return FAQ_OK;
  if (w4s::small_m_fits(m, k)) {  // a few rows: the weight streams packed into register-fragment MMAs
    const w4s::Params sp{static_cast<const __nv_bfloat16*>(a), lda, b_codes, b_meta, static_cast<int>(m),
                         static_cast<int>(n), static_cast<int>(k), static_cast<const __nv_bfloat16*>(bias),
                         static_cast<const __nv_bfloat16*>(residual), ldr, static_cast<__nv_bfloat16*>(y), ldy};
    return w4s::launch_small_m(sp, stream);
  }
  const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
  const uint64_t strides[1] = {static_cast<uint64_t>(lda) * 2};
  const uint32_t box[2] = {w4a4::BK, 128};
  rc = make_tmap(&maps.a_bf16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != FAQ_OK) return rc;
  return w4a4::launch(maps, false, p, stream);
}
