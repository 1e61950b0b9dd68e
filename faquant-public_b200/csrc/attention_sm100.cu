// K5 -- HiF4 QK/PV flash attention on tcgen05 tensor cores.
//
// Semantics (simulated_flash_attention.py:457-909, key chunk 128; Wan's Triton kernel
// wan22_attention.py:105-162): key tiles of 128 in order, fp32 scores times `scale`,
// bottom-right causal mask, online softmax against the running max that includes
// the current tile, P = exp(s - max) HiF4-quantized (unsigned) along the tile's keys
// in two groups of 64, the denominator from the quantized P (P-Reordering) or the
// raw P, O = alpha * O + P.V, out = O / denominator. Fully-future tiles are skipped
// (bitwise identical, simulated_flash_attention.py:676-699).
//
// One CTA per (128-query tile, q head, batch), 192 threads:
//   warp 0      TMA producer: Q [128 x 128] once, then K and V tiles [128 x 128]
//               (two 64-column 128-byte-swizzled chunks each) into a 2-stage ring;
//   warp 1      TMEM allocation (512 columns: S0, S1, O) and the single MMA-issuing
//               lane: S[j%2] = Q.K_j^T (M=N=128, 8 x K=16), then O += P_j.V_j with V
//               as an MN-major operand; tcgen05.commit signals the consumers;
//   warps 2..5  one query row per thread: tcgen05.ld of the S row, mask, running max,
//               exp2, HiF4 quantization of both 64-key groups inside the thread, the
//               row sum, P written to shared memory in the swizzled K-major layout the
//               MMA reads, O rescaled in TMEM when the max moved (alpha != 1), and at
//               the end O / denominator stored as bf16.
// The QK^T of tile j+1 runs on the tensor cores while tile j is in softmax. Every wait
// is bounded (common.cuh).
#include <algorithm>

#include "common.cuh"
#include "hif4.cuh"
#include "tma.h"

namespace faq {
namespace attn {

constexpr int BM = 128;   // queries per CTA
constexpr int BN = 128;   // keys per tile
constexpr int D = 128;    // head dim
constexpr int THREADS = 192;
constexpr int TILE_BYTES = BM * D * 2;      // 32 KB (two 16 KB chunks)
constexpr int CHUNK_BYTES = 128 * 128;      // 128 rows x 128 B
constexpr int KV_STAGES = 2;
constexpr uint32_t IDESC_QK = idesc_bf16_f32(BM, BN, false, false);
constexpr uint32_t IDESC_PV = idesc_bf16_f32(BM, D, false, true);
constexpr int TMEM_COLS = 512;
constexpr int S_COL0 = 0, O_COL = 256;
// smem: Q | K[2] | V[2] | P | barriers
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + TILE_BYTES;
constexpr int OFF_V = OFF_K + KV_STAGES * TILE_BYTES;
constexpr int OFF_P = OFF_V + KV_STAGES * TILE_BYTES;
constexpr int OFF_BAR = OFF_P + BM * BN * 2;
constexpr size_t SMEM_BYTES = 1024 + OFF_BAR + 256;

struct Params {
  int64_t sq, sk;
  int hq, hkv, group;  // group = hq / hkv
  int m_tiles;
  float scale_log2;    // scale * log2(e)
  int causal;
  int p_levels;        // 0: P not quantized
  int norm_quantized;
  __nv_bfloat16* out;
  int64_t ob, os, oh;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// HiF4 quantization (unsigned) of one 64-key group held by this thread, in place;
// returns the sum of the quantized values. Same arithmetic as hif4_quant8.
__device__ __forceinline__ float quantize_p64(float* p, int levels) {
  float m3[16], m2[8];
#pragma unroll
  for (int i = 0; i < 16; ++i) m3[i] = fmaxf(fmaxf(p[4 * i], p[4 * i + 1]), fmaxf(p[4 * i + 2], p[4 * i + 3]));
#pragma unroll
  for (int i = 0; i < 8; ++i) m2[i] = fmaxf(m3[2 * i], m3[2 * i + 1]);
  float m1 = m2[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) m1 = fmaxf(m1, m2[i]);
  const Hif4Scale sc = hif4_scale(m1, levels);
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int lv2 = 0, lv3a = 0, lv3b = 0;
    if (levels == 123) {
      lv2 = __fmul_rn(m2[i], sc.rec) >= 4.0f;
      const float thr = lv2 ? 4.0f : 2.0f;
      lv3a = __fmul_rn(m3[2 * i], sc.rec) >= thr;
      lv3b = __fmul_rn(m3[2 * i + 1], sc.rec) >= thr;
    } else if (levels == 12) {
      lv2 = __fmul_rn(m2[i], sc.rec) >= 2.0f;
    } else {
      lv3a = __fmul_rn(m3[2 * i], sc.rec) >= 2.0f;
      lv3b = __fmul_rn(m3[2 * i + 1], sc.rec) >= 2.0f;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int sh = lv2 + (h ? lv3b : lv3a);
      const float qm4 = __fmul_rn(sc.rec, pow2f(2 - sh));  // 4 * qm, exact
      const float ds4 = __fmul_rn(sc.s, pow2f(sh - 2));
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        float& v = p[8 * i + 4 * h + t];
        v = __fmul_rn(hif4_code4(v, qm4), ds4);
        sum = __fadd_rn(sum, v);
      }
    }
  }
  return sum;
}

__global__ void __launch_bounds__(THREADS, 1)
    hif4_attention_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                          const __grid_constant__ CUtensorMap tmap_v, Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_empty = bars + 11; // [2]
  uint64_t* p_full = bars + 13;
  uint64_t* o_done = bars + 14;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // longest causal rows first: the last query tile has the most key tiles
  const int m_tile = p.causal ? (p.m_tiles - 1 - static_cast<int>(blockIdx.x)) : static_cast<int>(blockIdx.x);
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / p.group;
  const int64_t q0 = static_cast<int64_t>(m_tile) * BM;
  const int64_t offset = p.sk - p.sq;  // bottom-right causal alignment
  int64_t kv_end = p.sk;
  if (p.causal) kv_end = std::min<int64_t>(p.sk, q0 + BM - 1 + offset + 1);
  const int n_tiles = kv_end <= 0 ? 0 : static_cast<int>((kv_end + BN - 1) / BN);

  if (threadIdx.x == 0) {
    mbar_init(smem_addr(q_full), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_addr(&k_full[i]), 1);
      mbar_init(smem_addr(&k_empty[i]), 1);
      mbar_init(smem_addr(&v_full[i]), 1);
      mbar_init(smem_addr(&v_empty[i]), 1);
      mbar_init(smem_addr(&s_full[i]), 1);
      mbar_init(smem_addr(&s_empty[i]), 4);
    }
    mbar_init(smem_addr(p_full), 4);
    mbar_init(smem_addr(o_done), 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n_tiles > 0) {
      bool ok = true;
      mbar_arrive_expect_tx(smem_addr(q_full), TILE_BYTES);
      for (int c = 0; c < 2; ++c)
        tma_load_4d(smem_addr(base + OFF_Q + c * CHUNK_BYTES), &tmap_q, smem_addr(q_full), c * 64,
                    static_cast<int>(q0), h, b);
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = ((j >> 1) & 1) ^ 1;
        if (!mbar_wait_site(smem_addr(&k_empty[st]), ph, 1, j)) { ok = false; break; }
        mbar_arrive_expect_tx(smem_addr(&k_full[st]), TILE_BYTES);
        for (int c = 0; c < 2; ++c)
          tma_load_4d(smem_addr(base + OFF_K + st * TILE_BYTES + c * CHUNK_BYTES), &tmap_k, smem_addr(&k_full[st]),
                      c * 64, j * BN, hk, b);
        if (!mbar_wait_site(smem_addr(&v_empty[st]), ph, 2, j)) { ok = false; break; }
        mbar_arrive_expect_tx(smem_addr(&v_full[st]), TILE_BYTES);
        for (int c = 0; c < 2; ++c)
          tma_load_4d(smem_addr(base + OFF_V + st * TILE_BYTES + c * CHUNK_BYTES), &tmap_v, smem_addr(&v_full[st]),
                      c * 64, j * BN, hk, b);
      }
      // drain (bounded): every load landed and was consumed before the CTA exits
      if (ok) {
        for (int j = std::max(0, n_tiles - 2); j < n_tiles; ++j) {
          const int st = j & 1;
          const uint32_t ph = (j >> 1) & 1;
          if (!mbar_wait_site(smem_addr(&k_empty[st]), ph, 3, j)) break;
          if (!mbar_wait_site(smem_addr(&v_empty[st]), ph, 3, j)) break;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_tiles > 0) {
      bool ok = mbar_wait_site(smem_addr(q_full), 0, 4, 0);
      const uint32_t q_base = smem_addr(base + OFF_Q);
      auto issue_qk = [&](int j) -> bool {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait_site(smem_addr(&k_full[st]), ph, 5, j)) return false;
        if (!mbar_wait_site(smem_addr(&s_empty[st]), ph ^ 1, 6, j)) return false;
        tc_fence_after();
        const uint32_t k_base = smem_addr(base + OFF_K + st * TILE_BYTES);
        const uint32_t d_tmem = tmem + S_COL0 + st * BN;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * CHUNK_BYTES + (kk & 3) * 32;
          tc_mma_f16(d_tmem, sw128_kmajor_desc(q_base + off), sw128_kmajor_desc(k_base + off), IDESC_QK, kk != 0);
        }
        tc_commit(smem_addr(&s_full[st]));
        tc_commit(smem_addr(&k_empty[st]));
        return true;
      };
      if (ok) ok = issue_qk(0);
      for (int j = 0; j < n_tiles && ok; ++j) {
        if (j + 1 < n_tiles && !issue_qk(j + 1)) break;
        const int st = j & 1;
        if (!mbar_wait_site(smem_addr(p_full), j & 1, 7, j)) break;
        if (!mbar_wait_site(smem_addr(&v_full[st]), (j >> 1) & 1, 8, j)) break;
        tc_fence_after();
        const uint32_t p_base = smem_addr(base + OFF_P);
        const uint32_t v_base = smem_addr(base + OFF_V + st * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // A = P [128 q x 128 keys] K-major: chunk kk/4, +32 B per 16 keys
          const uint32_t a_off = (kk >> 2) * CHUNK_BYTES + (kk & 3) * 32;
          // B = V [128 keys x 128 d] MN-major: 16 key rows = 2048 B per step
          tc_mma_f16(tmem + O_COL, sw128_kmajor_desc(p_base + a_off), sw128_mnmajor_desc(v_base + kk * 2048, CHUNK_BYTES),
                     IDESC_PV, (j | kk) != 0);
        }
        tc_commit(smem_addr(o_done));
        tc_commit(smem_addr(&v_empty[st]));
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax warps
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;          // TMEM lane == query row in tile
    const int64_t qpos = q0 + row;                // query index
    const int64_t anchor = qpos + offset;         // last visible key (causal)
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    float m_run = -INFINITY, l_run = 0.0f;
    uint8_t* p_row = base + OFF_P + row * 128;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      if (!mbar_wait_warp(smem_addr(&s_full[st]), (j >> 1) & 1, 9, j)) { ok = false; break; }
      tc_fence_after();
      float s[BN];
      {
        uint32_t r0[32], r1[32], r2[32], r3[32];
        const uint32_t sa = tmem + lane_addr + S_COL0 + st * BN;
        tmem_ld32(sa, r0);
        tmem_ld32(sa + 32, r1);
        tmem_ld32(sa + 64, r2);
        tmem_ld32(sa + 96, r3);
        tc_wait_ld();
        reg_fence32(r0);
        reg_fence32(r1);
        reg_fence32(r2);
        reg_fence32(r3);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = __uint_as_float(r0[i]);
          s[32 + i] = __uint_as_float(r1[i]);
          s[64 + i] = __uint_as_float(r2[i]);
          s[96 + i] = __uint_as_float(r3[i]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&s_empty[st]));
      // scores in the log2 domain; mask future / out-of-range keys
      const int64_t key0 = static_cast<int64_t>(j) * BN;
      const bool need_mask = (key0 + BN > p.sk) || (p.causal && key0 + BN - 1 > q0 + offset);
      float tmax = -INFINITY;
#pragma unroll
      for (int i = 0; i < BN; ++i) {
        float t = __fmul_rn(s[i], p.scale_log2);
        if (need_mask) {
          const int64_t key = key0 + i;
          if (key >= p.sk || (p.causal && key > anchor)) t = -INFINITY;
        }
        s[i] = t;
        tmax = fmaxf(tmax, t);
      }
      const float m_new = fmaxf(m_run, tmax);
      const float m_use = m_new == -INFINITY ? 0.0f : m_new;
      const float alpha = m_run == -INFINITY ? 0.0f : ex2(__fsub_rn(m_run, m_use));
      float raw_sum = 0.0f;
#pragma unroll
      for (int i = 0; i < BN; ++i) {
        s[i] = ex2(__fsub_rn(s[i], m_use));
        raw_sum = __fadd_rn(raw_sum, s[i]);
      }
      float q_sum = raw_sum;
      if (p.p_levels != 0) q_sum = __fadd_rn(quantize_p64(s, p.p_levels), quantize_p64(s + 64, p.p_levels));
      l_run = __fadd_rn(__fmul_rn(alpha, l_run), p.norm_quantized ? q_sum : raw_sum);
      m_run = m_new;
      // P and O may be touched only after PV of the previous tile finished
      if (j > 0) {
        if (!mbar_wait_warp(smem_addr(o_done), (j - 1) & 1, 10, j)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tmem + lane_addr + O_COL + c * 32, r);
            tc_wait_ld();
            reg_fence32(r);
            float o[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __fmul_rn(__uint_as_float(r[i]), alpha);
            tmem_st32(tmem + lane_addr + O_COL + c * 32, o);
          }
          tc_wait_st();
        }
      }
      // P (bf16, exact for quantized values) into the 128-byte swizzled K-major layout
#pragma unroll
      for (int c = 0; c < 2; ++c) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float* v = s + c * 64 + u * 8;
          uint32_t w[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const __nv_bfloat162 pr = __floats2bfloat162_rn(v[2 * t], v[2 * t + 1]);
            w[t] = *reinterpret_cast<const uint32_t*>(&pr);
          }
          const int phys = u ^ (row & 7);
          *reinterpret_cast<uint4*>(p_row + c * CHUNK_BYTES + phys * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(p_full));
    }
    if (ok && n_tiles > 0 && mbar_wait_warp(smem_addr(o_done), (n_tiles - 1) & 1, 11, n_tiles)) {
      tc_fence_after();
      // tcgen05.ld is .sync.aligned: every lane of the warp loads, even the lanes of
      // query rows past the end (a tile can end mid-warp); only the stores are predicated.
      const bool store = qpos < p.sq;
      __nv_bfloat16* dst = p.out + b * p.ob + (store ? qpos : 0) * p.os + static_cast<int64_t>(h) * p.oh;
      const bool has_mass = l_run > 0.0f;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_addr + O_COL + c * 32, r);
        tc_wait_ld();
        reg_fence32(r);
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float a0 = has_mass ? __fdiv_rn(__uint_as_float(r[2 * i]), l_run) : 0.0f;
          const float a1 = has_mass ? __fdiv_rn(__uint_as_float(r[2 * i + 1]), l_run) : 0.0f;
          const __nv_bfloat162 pr = __floats2bfloat162_rn(a0, a1);
          w[i] = *reinterpret_cast<const uint32_t*>(&pr);
        }
        if (store) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) d4[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
    } else if (n_tiles == 0 && qpos < p.sq) {
      // no visible key at all: the reference's output is zero
      __nv_bfloat16* dst = p.out + b * p.ob + qpos * p.os + static_cast<int64_t>(h) * p.oh;
      for (int i = 0; i < D; ++i) dst[i] = __float2bfloat16_rn(0.0f);
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
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
  p.m_tiles = static_cast<int>((sq + BM - 1) / BM);
  p.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);
  p.causal = causal;
  p.p_levels = p_levels;
  p.norm_quantized = normalizer_quantized;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ob = ob;
  p.os = os;
  p.oh = oh;
  FAQ_CUDA(cudaFuncSetAttribute(hif4_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(SMEM_BYTES)));
  dim3 grid(p.m_tiles, static_cast<unsigned>(hq), static_cast<unsigned>(batch));
  hif4_attention_kernel<<<grid, THREADS, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, p);
  return launch_status("hif4_attention_kernel");
}
