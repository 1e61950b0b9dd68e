// K5 -- HiF4 QK/PV flash attention on tcgen05 tensor cores.
//
// Semantics (simulated_flash_attention.py:457-909, key chunk 128; Wan's Triton kernel
// wan22_attention.py:105-162): key tiles of 128 in order, fp32 scores times `scale`,
// bottom-right causal mask, online softmax against the running max that includes
// the current tile, P = exp(s - max) HiF4-quantized (unsigned) along the tile's keys
// in two groups of 64, the denominator from the quantized P (P-Reordering) or the
// raw P, O = alpha * O + P.V, out = O / denominator.
//
// One CTA per (256 queries = two 128-query tiles A and B, q head, batch), 640 threads
// in five warpgroups; setmaxnreg moves registers from the fifth to the first four
// (launch 96 x 640 = 112 x 512 + 32 x 128, exactly):
//   warps 0..7   softmax of tile A, warps 8..15 softmax of tile B; within a tile the
//                first four warps take keys 0..63 of every key tile and the other four
//                keys 64..127 -- one HiF4 group each -- for the same query rows (a
//                warp reaches the tensor-memory lanes 32 (warp % 4) .. + 31);
//   warp 16      TMA producer of Q_A and Q_B (once) and of the K tiles [128 x 128] (two
//                64-column 128-byte-swizzled chunks) into a 2-stage ring;
//   warp 17      TMEM allocation (512 columns: S_A, S_B, O_A, O_B) and the single
//                MMA-issuing lane: S_t = Q_t.K_j^T and O_t += P_t.V_j, both SS form (P is
//                written by the softmax warps to shared memory in the layout TMA gives
//                Q; V is an MN-major operand);
//   warp 18      TMA producer of the V tiles (one stage);
//   warp 19      no role.
// Softmax, per key tile and query row, split over the two key halves: tcgen05.ld of the
// half row of S and, for the row maximum only, of the other half (no exchange between
// the warps); as soon as S is in registers the tile's eight warps release it and the
// tensor core computes the next S_t = Q_t.K_{j+1}^T while they work. Then mask, max,
// exp2 and HiF4 quantization of the half's 64-key group on FP32x2 pairs, interleaved by
// 8-key sub-block (the group's scale comes from the largest score), a running sum per
// half (same maxima, so the two sums add up at the end); once PV_t(j-1) has completed,
// P goes to shared memory and this half's 64 columns of O are rescaled when the max moved
// (alpha == 1 is exact and skipped); at the end O / (sum_0 + sum_1). The two tiles
// share the tensor core; with causal masking both walk the key tiles of tile B, the
// extra tile of tile A being fully masked (P = 0, alpha = 1: no effect).
// Every wait is bounded (common.cuh) and warp-uniform for whole-warp roles.
#include <algorithm>

#include "common.cuh"
#include "hif4.cuh"
#include "tma.h"

namespace faq {
namespace attn {

constexpr int BM = 128;   // queries per tile
constexpr int BN = 128;   // keys per tile
constexpr int D = 128;    // head dim
constexpr int THREADS = 640;
constexpr int SOFTMAX_WARPS = 16;
constexpr int PRODUCER_WARP = 16, MMA_WARP = 17, V_WARP = 18;
constexpr int TILE_BYTES = BM * D * 2;      // 32 KB (two 16 KB chunks)
constexpr int CHUNK_BYTES = 128 * 128;      // 128 rows x 128 B
constexpr int K_STAGES = 2;
constexpr uint32_t IDESC_QK = idesc_bf16_f32(BM, BN, false, false);
constexpr uint32_t IDESC_PV = idesc_bf16_f32(BM, D, false, true);
constexpr int TMEM_COLS = 512;
__device__ __forceinline__ uint32_t s_col(int t) { return t ? 128u : 0u; }
__device__ __forceinline__ uint32_t o_col(int t) { return t ? 384u : 256u; }
// smem: Q_A | Q_B | K[2] | V[2] | row exchange [2 parities][2 tiles][2 halves][128] f32 | barriers
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + 2 * TILE_BYTES;
constexpr int OFF_V = OFF_K + K_STAGES * TILE_BYTES;
constexpr int OFF_P = OFF_V + TILE_BYTES;  // P_A, P_B; after the last PV, the row sums' exchange
constexpr int OFF_BAR = OFF_P + 2 * TILE_BYTES;
constexpr size_t SMEM_BYTES = 1024 + OFF_BAR + 256;

// Named barrier over the `count` threads of one tile's softmax warps that also ANDs a
// predicate across them (bar.red orders their shared-memory accesses like bar.sync).
__device__ __forceinline__ bool bar_and(int id, int count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void st_shared_f32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ float ld_shared_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

struct Params {
  int64_t sq, sk;
  int hq, hkv, group;  // group = hq / hkv
  int m_tiles;         // CTAs along the queries (256 queries each)
  float scale_log2;    // scale * log2(e)
  int causal;
  int p_levels;        // 0: P not quantized
  int norm_quantized;
  __nv_bfloat16* out;
  int64_t ob, os, oh;
};

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// HiF4 quantization (unsigned) of one 64-key group held by this thread (f[0..63]), in
// place; returns the sum of the quantized values. The same arithmetic as hif4_quant8,
// rearranged only where exact, on FP32x2 pairs:
//   t = min(fl(fl(p * 4qm) + 0.5), 7.5)      (== the reference's clamp of the code to 7)
//   r = t + 2^23 rounded toward zero          (== 2^23 + floor(t))
//   q = fma(r, ds/4, -2^23 * ds/4)           (exact: the result code * ds/4 has <= 6 bits)
// Maxima and the sum are trees, so the dependency chains stay short.
template <int LEVELS>
__device__ __forceinline__ float quantize_p64(float* f) {
  float m3[16], m2[8];
#pragma unroll
  for (int i = 0; i < 16; ++i) m3[i] = fmaxf(fmaxf(f[4 * i], f[4 * i + 1]), fmaxf(f[4 * i + 2], f[4 * i + 3]));
#pragma unroll
  for (int i = 0; i < 8; ++i) m2[i] = fmaxf(m3[2 * i], m3[2 * i + 1]);
  const float m1 = fmaxf(fmaxf(fmaxf(m2[0], m2[1]), fmaxf(m2[2], m2[3])), fmaxf(fmaxf(m2[4], m2[5]), fmaxf(m2[6], m2[7])));
  const Hif4Scale sc = hif4_scale(m1, LEVELS);
  float2 part[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t ea, eb;
    hif4_level_shifts(__fmul_rn(m3[2 * i], sc.rec), __fmul_rn(m3[2 * i + 1], sc.rec), LEVELS, ea, eb);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int sh = static_cast<int>((h ? eb : ea) >> 23);
      const float qm4 = __fmul_rn(sc.rec, pow2f(2 - sh));  // 4 * qm, exact
      const float ds4 = __fmul_rn(sc.s, pow2f(sh - 2));    // ds / 4, exact
      const float2 qm2 = make_float2(qm4, qm4), ds2 = make_float2(ds4, ds4);
      const float2 off2 = make_float2(-8388608.0f * ds4, -8388608.0f * ds4);
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        float* v = f + 8 * i + 4 * h + 2 * t;
        float2 y = __fadd2_rn(__fmul2_rn(make_float2(v[0], v[1]), qm2), make_float2(0.5f, 0.5f));
        y = make_float2(fminf(y.x, 7.5f), fminf(y.y, 7.5f));
        const float2 r = __fadd2_rz(y, make_float2(8388608.0f, 8388608.0f));
        const float2 q = __ffma2_rn(r, ds2, off2);
        v[0] = q.x;
        v[1] = q.y;
        part[2 * h + t] = __fadd2_rn(part[2 * h + t], q);
      }
    }
  }
  const float2 s01 = __fadd2_rn(part[0], part[1]), s23 = __fadd2_rn(part[2], part[3]);
  const float2 s = __fadd2_rn(s01, s23);
  return __fadd_rn(s.x, s.y);
}

// 2^(lv2 + lv3) of the two quarters of an 8-key sub-block of P, as floats, from the
// products r = (fl(m3a * rec), fl(m3b * rec)) of the quarter maxima with the group's
// reciprocal: hif4_level_shifts' comparisons for products that are finite, non-negative
// and below 8 (levels 123) or 4 (12, 13). P is in [0, 1], so the E6M2 scale of its group
// is not clamped from above, and m3 * rec <= max / s <= 1.125 * 7.0137 * (1 + 2^-9) < 7.91
// for the divisor 7 (tie-to-even E6M2 rounding lowers s by at most a factor 1.125; 1/7 and
// 1/s are bf16-rounded), half that for the divisor 3.5: the exponent comparisons reduce to
// maxima of powers of two, without the upper clamps. 2^floor(log2 r) is r's exponent field
// (0 for r = 0), lv2 (123) is [max(r) >= 4], so 2^lv2 = max(2^floor(log2 max(r)) / 2, 1) and
// 2^(lv2 + lv3) = max(2^floor(log2 r), 2^lv2). A NaN product (a quarter of NaN scores) gives
// other shifts, but its row's output is NaN whatever they are.
template <int LEVELS>
__device__ __forceinline__ float2 p_shift_pow2(float2 r) {
  const float pa = __uint_as_float(__float_as_uint(r.x) & 0x7F800000u);
  const float pb = __uint_as_float(__float_as_uint(r.y) & 0x7F800000u);
  if constexpr (LEVELS == 123) {
    const float2 h = __fmul2_rn(make_float2(pa, pb), make_float2(0.5f, 0.5f));
    const float lv = fmax3(h.x, h.y, 1.0f);
    return make_float2(fmaxf(pa, lv), fmaxf(pb, lv));
  } else if constexpr (LEVELS == 12) {
    const float e = fmax3(pa, pb, 1.0f);
    return make_float2(e, e);
  } else {
    return make_float2(fmaxf(pa, 1.0f), fmaxf(pb, 1.0f));
  }
}

// exp2 and HiF4 quantization of one 64-key group (this thread's half row, f[0..63] the
// masked scores), sub-block by sub-block so that the exp2 of one sub-block overlaps the
// quantization of the previous one. p = ex2(fma(s, c, -m)) as in the unfused form; the
// group maximum is taken from the scores: p_max = ex2(fma(s_max, c, -m)) is the largest
// p, since fma with c > 0 and ex2.approx.ftz are both non-decreasing (the second checked
// over every float in [-inf, 1] on the device, faq_selftest_ex2_monotone). Returns the
// sum of the quantized values; *raw gets the sum of the unquantized p.
template <int LEVELS, bool RAW>
__device__ __forceinline__ float exp_quantize_p64(float* f, float2 c2, float2 mneg, float s_max, float* raw) {
  const float m1 = ex2(__fmaf_rn(s_max, c2.x, mneg.x));
  const Hif4Scale sc = hif4_scale(m1, LEVELS);
  const float2 rec2 = make_float2(sc.rec, sc.rec);
  // with w = 2^sh: 4 qm = rec * 2^(2 - sh) by an exponent move (bits(w) = (127 + sh) << 23),
  // ds / 4 = (s / 4) * w and -2^23 ds / 4 = (-2^23 s / 4) * w, exact products
  const uint32_t rec_w = __float_as_uint(sc.rec) + (2u << 23) + 0x3F800000u;
  const float s_q = __uint_as_float(__float_as_uint(sc.s) - (2u << 23));
  const float2 sq2 = make_float2(s_q, s_q), so2 = make_float2(-8388608.0f * s_q, -8388608.0f * s_q);
  float2 part[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
  float2 rp[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float* v = f + 8 * i;
    float2 e[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 d = __ffma2_rn(make_float2(v[2 * t], v[2 * t + 1]), c2, mneg);  // s * c - m, one rounding
      e[t] = make_float2(ex2(d.x), ex2(d.y));
      if constexpr (RAW) rp[t] = __fadd2_rn(rp[t], e[t]);
    }
    const float m3a = fmaxf(fmax3(e[0].x, e[0].y, e[1].x), e[1].y);
    const float m3b = fmaxf(fmax3(e[2].x, e[2].y, e[3].x), e[3].y);
    const float2 rab = __fmul2_rn(make_float2(m3a, m3b), rec2);
    const float2 w = p_shift_pow2<LEVELS>(rab);
    const float qa = __uint_as_float(rec_w - __float_as_uint(w.x)), qb = __uint_as_float(rec_w - __float_as_uint(w.y));
    const float2 dd = __fmul2_rn(w, sq2), oo = __fmul2_rn(w, so2);
    const float da = dd.x, db = dd.y, oa = oo.x, ob = oo.y;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float qm = t < 2 ? qa : qb, ds = t < 2 ? da : db, off = t < 2 ? oa : ob;
      float2 y = __fadd2_rn(__fmul2_rn(e[t], make_float2(qm, qm)), make_float2(0.5f, 0.5f));
      y = make_float2(fminf(y.x, 7.5f), fminf(y.y, 7.5f));
      const float2 r = __fadd2_rz(y, make_float2(8388608.0f, 8388608.0f));
      const float2 q = __ffma2_rn(r, make_float2(ds, ds), make_float2(off, off));
      v[2 * t] = q.x;
      v[2 * t + 1] = q.y;
      part[t] = __fadd2_rn(part[t], q);
    }
  }
  if constexpr (RAW) {
    const float2 r = __fadd2_rn(__fadd2_rn(rp[0], rp[1]), __fadd2_rn(rp[2], rp[3]));
    *raw = __fadd_rn(r.x, r.y);
  }
  const float2 s = __fadd2_rn(__fadd2_rn(part[0], part[1]), __fadd2_rn(part[2], part[3]));
  return __fadd_rn(s.x, s.y);
}

// PLEV: HiF4 levels of P (0 = P not quantized); RAW: the denominator sums the raw P
template <int PLEV, bool RAW>
__global__ void __launch_bounds__(THREADS, 1)
    hif4_attention_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                          const __grid_constant__ CUtensorMap tmap_v, Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;
  uint64_t* v_empty = bars + 6;
  uint64_t* s_full = bars + 7;   // [2 tiles] S_t(j) computed
  uint64_t* s_free = bars + 9;   // [2 tiles] S_t(j) read by the tile's eight warps
  uint64_t* p_full = bars + 11;  // [2 tiles] P_t(j) written, O_t rescaled
  uint64_t* p_free = bars + 13;  // [2 tiles] PV_t(j) completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // longest causal rows first: the last query tiles have the most key tiles
  const int m_tile = p.causal ? (p.m_tiles - 1 - static_cast<int>(blockIdx.x)) : static_cast<int>(blockIdx.x);
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / p.group;
  const int64_t q0 = static_cast<int64_t>(m_tile) * (2 * BM);
  const int64_t offset = p.sk - p.sq;  // bottom-right causal alignment
  int64_t kv_end = p.sk;
  if (p.causal) kv_end = std::min<int64_t>(p.sk, q0 + 2 * BM - 1 + offset + 1);
  const int n_tiles = kv_end <= 0 ? 0 : static_cast<int>((kv_end + BN - 1) / BN);

  if (threadIdx.x == 0) {
    mbar_init(smem_addr(q_full), 1);
    mbar_init(smem_addr(v_full), 1);
    mbar_init(smem_addr(v_empty), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_addr(&k_full[i]), 1);
      mbar_init(smem_addr(&k_empty[i]), 1);
      mbar_init(smem_addr(&s_full[i]), 1);
      mbar_init(smem_addr(&s_free[i]), 8);  // the eight softmax warps of the tile
      mbar_init(smem_addr(&p_full[i]), 8);
      mbar_init(smem_addr(&p_free[i]), 1);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
  }
  if (warp == MMA_WARP) {
    tmem_alloc(smem_addr(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Register split by warpgroup. The setmaxnreg of a role sits at the top of that
  // role's own branch: code after a merge point is compiled for the smaller budget.
  if (warp >= SOFTMAX_WARPS) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 32;\n" ::: "memory");
    if (warp == PRODUCER_WARP) {
    // ------------------------------------------------------------ Q and K producer
    if (lane == 0 && n_tiles > 0) {
      bool ok = true;
      mbar_arrive_expect_tx(smem_addr(q_full), 2 * TILE_BYTES);
      for (int t = 0; t < 2; ++t)
        for (int c = 0; c < 2; ++c)
          tma_load_4d(smem_addr(base + OFF_Q + t * TILE_BYTES + c * CHUNK_BYTES), &tmap_q, smem_addr(q_full), c * 64,
                      static_cast<int>(q0 + t * BM), h, b);
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait_site(smem_addr(&k_empty[st]), ((j >> 1) & 1) ^ 1, 1, j)) { ok = false; break; }
        mbar_arrive_expect_tx(smem_addr(&k_full[st]), TILE_BYTES);
        for (int c = 0; c < 2; ++c)
          tma_load_4d(smem_addr(base + OFF_K + st * TILE_BYTES + c * CHUNK_BYTES), &tmap_k, smem_addr(&k_full[st]),
                      c * 64, j * BN, hk, b);
      }
      // drain (bounded): every load landed and was consumed before the CTA exits
      if (ok) {
        for (int j = std::max(0, n_tiles - 2); j < n_tiles; ++j)
          if (!mbar_wait_site(smem_addr(&k_empty[j & 1]), (j >> 1) & 1, 3, j)) break;
      }
    }
    __syncwarp();
    } else if (warp == V_WARP) {
    // ------------------------------------------------------------ V producer
    if (lane == 0 && n_tiles > 0) {
      bool ok = true;
      for (int j = 0; j < n_tiles && ok; ++j) {
        if (!mbar_wait_site(smem_addr(v_empty), (j & 1) ^ 1, 2, j)) { ok = false; break; }
        mbar_arrive_expect_tx(smem_addr(v_full), TILE_BYTES);
        for (int c = 0; c < 2; ++c)
          tma_load_4d(smem_addr(base + OFF_V + c * CHUNK_BYTES), &tmap_v, smem_addr(v_full), c * 64, j * BN, hk, b);
      }
      if (ok) mbar_wait_site(smem_addr(v_empty), (n_tiles - 1) & 1, 3, n_tiles);
    }
    __syncwarp();
    } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_tiles > 0) {
      bool ok = mbar_wait_site(smem_addr(q_full), 0, 4, 0);
      // Shared-memory descriptors built once; every MMA adds a compile-time offset to a
      // base (the 14-bit start-address field holds addr >> 4 and cannot carry: shared
      // addresses stay below 2^18). Unrolled, so an MMA issues every few cycles instead
      // of waiting on a descriptor chain -- one N = 128 MMA runs only 64 cycles.
      const uint32_t q_desc = sw128_desc_lo(smem_addr(base + OFF_Q), 16);  // LBO unused (K-major SW128)
      const uint32_t k_desc = sw128_desc_lo(smem_addr(base + OFF_K), 16);
      const uint32_t p_desc = sw128_desc_lo(smem_addr(base + OFF_P), 16);
      const uint32_t v_desc = sw128_desc_lo(smem_addr(base + OFF_V), CHUNK_BYTES);
      constexpr uint32_t TILE_D = TILE_BYTES >> 4;
      // an opaque copy keeps the compiler from hoisting every per-MMA descriptor of the
      // loop into registers (the issuing warp runs on 32)
      auto pin = [](uint32_t v) {
        asm volatile("mov.b32 %0, %0;" : "+r"(v));
        return v;
      };
      // S_t = Q_t . K_j^T
      auto issue_qk = [&](int t, int j) {
        const uint32_t a = pin(q_desc + t * TILE_D), bq = pin(k_desc + (j & 1) * TILE_D);
        const uint32_t d = tmem + s_col(t);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = static_cast<uint32_t>((kk >> 2) * CHUNK_BYTES + (kk & 3) * 32) >> 4;
          tc_mma_f16_lo(d, a + off, bq + off, IDESC_QK, kk != 0);
        }
        tc_commit(smem_addr(&s_full[t]));
      };
      // O_t += P_t . V_j: P_t [128 queries x 128 keys] K-major like Q, V_j MN-major
      auto issue_pv = [&](int t, int j) {
        const uint32_t a = pin(p_desc + t * TILE_D), bv = pin(v_desc);
        const uint32_t d = tmem + o_col(t);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint32_t off = static_cast<uint32_t>((kk >> 2) * CHUNK_BYTES + (kk & 3) * 32) >> 4;
          tc_mma_f16_lo(d, a + off, bv + ((kk * 2048) >> 4), IDESC_PV, (j | kk) != 0);
        }
        tc_commit(smem_addr(&p_free[t]));
      };
      if (ok) ok = mbar_wait_site(smem_addr(&k_full[0]), 0, 5, 0);
      if (ok) {
        tc_fence_after();
        issue_qk(0, 0);
        issue_qk(1, 0);
        tc_commit(smem_addr(&k_empty[0]));
      }
      for (int j = 0; j < n_tiles && ok; ++j) {
        if (j + 1 < n_tiles) {
          // S_t(j + 1) as soon as the tile's warps hold S_t(j) in registers
          if (!mbar_wait_site(smem_addr(&k_full[(j + 1) & 1]), ((j + 1) >> 1) & 1, 5, j + 1)) break;
          if (!mbar_wait_site(smem_addr(&s_free[0]), j & 1, 6, j)) break;
          tc_fence_after();
          issue_qk(0, j + 1);
          if (!mbar_wait_site(smem_addr(&s_free[1]), j & 1, 7, j)) break;
          tc_fence_after();
          issue_qk(1, j + 1);
          tc_commit(smem_addr(&k_empty[(j + 1) & 1]));
        }
        if (!mbar_wait_site(smem_addr(v_full), j & 1, 8, j)) break;
        if (!mbar_wait_site(smem_addr(&p_full[0]), j & 1, 9, j)) break;
        tc_fence_after();
        issue_pv(0, j);
        if (!mbar_wait_site(smem_addr(&p_full[1]), j & 1, 10, j)) break;
        tc_fence_after();
        issue_pv(1, j);
        tc_commit(smem_addr(v_empty));
      }
    }
    __syncwarp();
    }  // warp 19 has no role
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 112;\n" ::: "memory");
    // ------------------------------------------------------------ softmax warps 0..15
    const int t = warp >> 3;                      // query tile of this warp
    const int hh = (warp >> 2) & 1;               // key half: keys 64 hh .. 64 hh + 63 of a key tile
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;          // TMEM lane == query row in the tile
    // Masking in 32 bits (sequence lengths are below 2^31, as the TMA coordinates are):
    // key tile j needs a mask in half x from j_mask[x] on, and the last visible key of
    // half x of tile j is lk[x] - 128 j (relative to the half's first key).
    int j_mask[2], lk[2];
    {
      const int64_t qpos = q0 + t * BM + row;
      const int64_t last_key = p.causal ? std::min<int64_t>(qpos + offset, p.sk - 1) : p.sk - 1;
      auto first_j = [](int64_t num) -> int64_t { return num < 0 ? 0 : num / BN + 1; };  // least j: BN j > num
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        int64_t jm = first_j(p.sk - 64 - 64 * x);  // keys past the end
        if (p.causal) jm = std::min<int64_t>(jm, first_j(q0 + t * BM + offset - 63 - 64 * x));  // future keys
        j_mask[x] = static_cast<int>(std::min<int64_t>(jm, n_tiles));
        lk[x] = static_cast<int>(std::max<int64_t>(-1, last_key - 64 * x));
      }
    }
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_addr + s_col(t) + 64 * hh;           // this half's S columns
    const uint32_t s_other = tmem + lane_addr + s_col(t) + 64 * (hh ^ 1);    // the other half's
    const uint32_t o_addr = tmem + lane_addr + o_col(t) + 64 * hh;           // this half's head dims of O
    // P_t in the 128-byte-swizzled K-major layout of a TMA tile: key chunk hh, row `row`,
    // 16-byte unit u of the row at u ^ (row % 8)
    const uint32_t p_row = smem_addr(base + OFF_P + t * TILE_BYTES + hh * CHUNK_BYTES + row * 128);
    const int p_sw = row & 7;
    const float2 c2 = make_float2(p.scale_log2, p.scale_log2);
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      if (!mbar_wait_warp(smem_addr(&s_full[t]), j & 1, 12 + t, j)) { ok = false; break; }
      float f[64];  // the half row of S, then P, in place
      float omax;
      tc_fence_after();
      {
        float g[32];
        tmem_ld32f(s_addr, f);
        tmem_ld32f(s_addr + 32, f + 32);
        tmem_ld32f(s_other, g);
        tc_wait_ld();
        reg_fence32f(f);
        reg_fence32f(f + 32);
        reg_fence32f(g);
        const int ho = hh ^ 1;
        if (j >= j_mask[ho]) {
          const int lim = std::max(-1, std::min(63, lk[ho] - BN * j));
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i > lim) g[i] = -INFINITY;
        }
        float m4[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) m4[q] = fmax3(g[8 * q], g[8 * q + 1], g[8 * q + 2]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          m4[q] = fmax3(m4[q], g[8 * q + 3], g[8 * q + 4]);
          m4[q] = fmax3(m4[q], g[8 * q + 5], g[8 * q + 6]);
          m4[q] = fmaxf(m4[q], g[8 * q + 7]);
        }
        tmem_ld32f(s_other + 32, g);
        tc_wait_ld();
        reg_fence32f(g);
        // S_t(j) is in registers: the tensor core may overwrite it with S_t(j + 1)
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&s_free[t]));
        if (j >= j_mask[ho]) {
          const int lim = std::max(-1, std::min(63, lk[ho] - BN * j));
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i + 32 > lim) g[i] = -INFINITY;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          m4[q] = fmax3(m4[q], g[8 * q], g[8 * q + 1]);
          m4[q] = fmax3(m4[q], g[8 * q + 2], g[8 * q + 3]);
          m4[q] = fmax3(m4[q], g[8 * q + 4], g[8 * q + 5]);
          m4[q] = fmax3(m4[q], g[8 * q + 6], g[8 * q + 7]);
        }
        omax = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      }
      // mask future / out-of-range keys; the max is taken on the raw scores (the scale is
      // positive, so max(fl(s * c)) == fl(max(s) * c))
      if (j >= j_mask[hh]) {
        const int lim = std::max(-1, std::min(63, lk[hh] - BN * j));
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i > lim) f[i] = -INFINITY;
      }
      float mx[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) mx[g] = fmax3(f[16 * g], f[16 * g + 1], f[16 * g + 2]);
#pragma unroll
      for (int g = 0; g < 4; ++g) {
#pragma unroll
        for (int i = 3; i < 15; i += 2) mx[g] = fmax3(mx[g], f[16 * g + i], f[16 * g + i + 1]);
        mx[g] = fmaxf(mx[g], f[16 * g + 15]);
      }
      const float own_max = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      const float tmax = fmaxf(own_max, omax);
      const float m_new = fmaxf(m_run, __fmul_rn(tmax, p.scale_log2));  // log2 domain
      const float m_use = m_new == -INFINITY ? 0.0f : m_new;
      const float alpha = m_run == -INFINITY ? 0.0f : ex2(__fsub_rn(m_run, m_use));
      const float2 mneg = make_float2(-m_use, -m_use);
      float half_sum;
      if constexpr (PLEV != 0) {
        float raw_sum = 0.0f;
        const float qs = exp_quantize_p64<PLEV, RAW>(f, c2, mneg, own_max, &raw_sum);
        half_sum = RAW ? raw_sum : qs;
      } else {
        float2 raw[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float2 d = __ffma2_rn(make_float2(f[2 * i], f[2 * i + 1]), c2, mneg);  // s * c - m, one rounding
          const float2 e = make_float2(ex2(d.x), ex2(d.y));
          f[2 * i] = e.x;
          f[2 * i + 1] = e.y;
          raw[i & 3] = __fadd2_rn(raw[i & 3], e);
        }
        const float2 r = __fadd2_rn(__fadd2_rn(raw[0], raw[1]), __fadd2_rn(raw[2], raw[3]));
        half_sum = __fadd_rn(r.x, r.y);
      }
      l_run = __fadd_rn(__fmul_rn(alpha, l_run), half_sum);
      m_run = m_new;
      // PV_t(j - 1) has completed: P_t may be overwritten and O_t is final for step j - 1
      if (j > 0 && !mbar_wait_warp(smem_addr(&p_free[t]), (j - 1) & 1, 14 + t, j)) { ok = false; break; }
      tc_fence_after();
      // P as bf16 (exact for quantized values), 16-byte units of 8 keys
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const __nv_bfloat162 pr = __floats2bfloat162_rn(f[8 * u + 2 * i], f[8 * u + 2 * i + 1]);
          w[i] = *reinterpret_cast<const uint32_t*>(&pr);
        }
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(p_row + ((u ^ p_sw) << 4)), "r"(w[0]),
                     "r"(w[1]), "r"(w[2]), "r"(w[3])
                     : "memory");
      }
      fence_proxy_async_smem();  // the tensor core reads P through the async proxy
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
        const float2 a2 = make_float2(alpha, alpha);
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          float o[32];
          tmem_ld32f(o_addr + c * 32, o);
          tc_wait_ld();
          reg_fence32f(o);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 v = __fmul2_rn(make_float2(o[2 * i], o[2 * i + 1]), a2);
            o[2 * i] = v.x;
            o[2 * i + 1] = v.y;
          }
          tmem_st32f(o_addr + c * 32, o);
        }
        tc_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&p_full[t]));
    }
    if (n_tiles > 0) {
      // every warp of the tile takes the barrier below once, whatever happened above
      const bool e_ok = ok && mbar_wait_warp(smem_addr(&p_free[t]), (n_tiles - 1) & 1, 16 + t, n_tiles);
      // the row sums of the two halves meet in P_t's buffer, free after the last PV_t
      const uint32_t red = smem_addr(base + OFF_P + t * TILE_BYTES);
      st_shared_f32(red + (hh * BM + row) * 4, l_run);
      if (bar_and(1 + t, 256, e_ok)) {
        tc_fence_after();
        const float l_sum = __fadd_rn(l_run, ld_shared_f32(red + ((hh ^ 1) * BM + row) * 4));
        const int64_t qpos = q0 + t * BM + row;
        // tcgen05.ld is .sync.aligned: every lane loads, even the lanes of query rows
        // past the end (a tile can end mid-warp); only the stores are predicated.
        const bool store = qpos < p.sq;
        __nv_bfloat16* dst = p.out + b * p.ob + (store ? qpos : 0) * p.os + static_cast<int64_t>(h) * p.oh + 64 * hh;
        const bool has_mass = l_sum > 0.0f;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          tmem_ld32(o_addr + c * 32, r);
          tc_wait_ld();
          reg_fence32(r);
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float a0 = has_mass ? __fdiv_rn(__uint_as_float(r[2 * i]), l_sum) : 0.0f;
            const float a1 = has_mass ? __fdiv_rn(__uint_as_float(r[2 * i + 1]), l_sum) : 0.0f;
            const __nv_bfloat162 pr = __floats2bfloat162_rn(a0, a1);
            w[i] = *reinterpret_cast<const uint32_t*>(&pr);
          }
          if (store) {
            uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) d4[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
          }
        }
      }
    } else if (q0 + t * BM + row < p.sq) {
      // no visible key at all: the reference's output is zero
      const int64_t qpos = q0 + t * BM + row;
      __nv_bfloat16* dst = p.out + b * p.ob + qpos * p.os + static_cast<int64_t>(h) * p.oh + 64 * hh;
      for (int i = 0; i < 64; ++i) dst[i] = __float2bfloat16_rn(0.0f);
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace attn
}  // namespace faq

extern "C" int faq_hif4_attention(const void* q, const void* k, const void* v, int64_t batch, int64_t hq, int64_t hkv,
                                  int64_t sq, int64_t sk, int d, int64_t qb, int64_t qh, int64_t qs, int64_t kb,
                                  int64_t kh, int64_t ks, int64_t vb, int64_t vh, int64_t vs, float scale, int causal,
                                  int p_levels, int normalizer_quantized, void* out, int64_t ob, int64_t os, int64_t oh,
                                  void* stream) {
  using namespace faq;
  using namespace faq::attn;
  FAQ_CHECK_ARG(q && k && v && out, "null pointer");
  FAQ_CHECK_ARG(batch >= 0 && hq > 0 && hkv > 0 && sq >= 0 && sk >= 0, "bad shape");
  FAQ_CHECK_ARG(sq < (int64_t(1) << 31) - 512 && sk < (int64_t(1) << 31) - 512,
                "sequence lengths must be below 2^31 - 512 (32-bit tile coordinates)");
  FAQ_CHECK_ARG(hq % hkv == 0, "query heads must be divisible by key/value heads");
  if (d != 128) return fail(FAQ_ERR_UNSUPPORTED, "head_dim must be 128");
  FAQ_CHECK_ARG(p_levels == 0 || p_levels == 123 || p_levels == 12 || p_levels == 13, "p_levels must be 0/123/12/13");
  FAQ_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out), "tensors must be 16-byte aligned");
  FAQ_CHECK_ARG(qb % 8 == 0 && qh % 8 == 0 && qs % 8 == 0 && kb % 8 == 0 && kh % 8 == 0 && ks % 8 == 0 &&
                    vb % 8 == 0 && vh % 8 == 0 && vs % 8 == 0 && ob % 8 == 0 && os % 8 == 0 && oh % 8 == 0,
                "strides must be multiples of 8 elements");
  FAQ_CHECK_ARG(sq < (int64_t(1) << 31) && sk < (int64_t(1) << 31) && hq < 65536 && batch < 65536, "shape too large");
  if (batch == 0 || sq == 0) return FAQ_OK;
  CUtensorMap tq, tk, tv;
  const uint32_t box[4] = {64, 128, 1, 1};
  {
    const uint64_t dims[4] = {128, static_cast<uint64_t>(sq), static_cast<uint64_t>(hq), static_cast<uint64_t>(batch)};
    const uint64_t str[3] = {static_cast<uint64_t>(qs) * 2, static_cast<uint64_t>(qh) * 2, static_cast<uint64_t>(qb) * 2};
    int rc = make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  const uint64_t skd = static_cast<uint64_t>(std::max<int64_t>(sk, 1));
  {
    const uint64_t dims[4] = {128, skd, static_cast<uint64_t>(hkv), static_cast<uint64_t>(batch)};
    const uint64_t str[3] = {static_cast<uint64_t>(ks) * 2, static_cast<uint64_t>(kh) * 2, static_cast<uint64_t>(kb) * 2};
    int rc = make_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, k, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[4] = {128, skd, static_cast<uint64_t>(hkv), static_cast<uint64_t>(batch)};
    const uint64_t str[3] = {static_cast<uint64_t>(vs) * 2, static_cast<uint64_t>(vh) * 2, static_cast<uint64_t>(vb) * 2};
    int rc = make_tmap(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, v, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  Params p;
  p.sq = sq;
  p.sk = sk;
  p.hq = static_cast<int>(hq);
  p.hkv = static_cast<int>(hkv);
  p.group = static_cast<int>(hq / hkv);
  p.m_tiles = static_cast<int>((sq + 2 * BM - 1) / (2 * BM));
  p.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);
  p.causal = causal;
  p.p_levels = p_levels;
  p.norm_quantized = normalizer_quantized;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ob = ob;
  p.os = os;
  p.oh = oh;
  const bool raw = !normalizer_quantized || p_levels == 0;
  auto kern = hif4_attention_kernel<123, false>;
  if (p_levels == 123) kern = raw ? hif4_attention_kernel<123, true> : hif4_attention_kernel<123, false>;
  else if (p_levels == 12) kern = raw ? hif4_attention_kernel<12, true> : hif4_attention_kernel<12, false>;
  else if (p_levels == 13) kern = raw ? hif4_attention_kernel<13, true> : hif4_attention_kernel<13, false>;
  else kern = hif4_attention_kernel<0, true>;
  FAQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(SMEM_BYTES)));
  dim3 grid(p.m_tiles, static_cast<unsigned>(hq), static_cast<unsigned>(batch));
  kern<<<grid, THREADS, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
  return launch_status("hif4_attention_kernel");
}

namespace faq {
namespace attn {
// ex2.approx.ftz over every float in [-inf, 1], in increasing order: counts the
// consecutive pairs whose results decrease (the group maximum of P above relies on none).
__device__ unsigned long long g_ex2_violations;
__device__ __forceinline__ uint32_t ordered_float_bits(uint64_t k) {
  constexpr uint64_t kNeg = 0xFF800000ull - 0x80000000ull + 1;  // -inf .. -0
  return k < kNeg ? static_cast<uint32_t>(0xFF800000ull - k) : static_cast<uint32_t>(k - kNeg);
}
__global__ void __launch_bounds__(256) ex2_monotone_kernel(uint64_t n) {
  unsigned long long bad = 0;
  for (uint64_t k = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; k + 1 < n;
       k += static_cast<uint64_t>(gridDim.x) * blockDim.x)
    bad += !(ex2(__uint_as_float(ordered_float_bits(k))) <= ex2(__uint_as_float(ordered_float_bits(k + 1))));
  if (bad) atomicAdd(&g_ex2_violations, bad);
}
}  // namespace attn
}  // namespace faq

extern "C" int faq_selftest_ex2_monotone(uint64_t* violations, void* stream) {
  using namespace faq;
  FAQ_CHECK_ARG(violations, "null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned long long zero = 0;
  FAQ_CUDA(cudaMemcpyToSymbolAsync(attn::g_ex2_violations, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, st));
  const uint64_t n = (0xFF800000ull - 0x80000000ull + 1) + 0x3F800000ull + 1;  // -inf .. +1.0
  attn::ex2_monotone_kernel<<<num_sms() * 8, 256, 0, st>>>(n);
  FAQ_CUDA(cudaGetLastError());
  unsigned long long bad = 0;
  FAQ_CUDA(cudaMemcpyFromSymbolAsync(&bad, attn::g_ex2_violations, sizeof(bad), 0, cudaMemcpyDeviceToHost, st));
  FAQ_CUDA(cudaStreamSynchronize(st));
  *violations = bad;
  return FAQ_OK;
}
