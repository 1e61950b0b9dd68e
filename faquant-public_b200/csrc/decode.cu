// K6 -- HiF4 attention decode (a few new query positions against a long K/V cache).
//
// Semantics are the prefill kernel's (K5) and the reference simulator's
// (simulated_flash_attention.py:623-884 with query_length <= 16): key tiles of 128 from
// key 0 in order, the running max including the current tile, P = exp(s - max)
// HiF4-quantized (unsigned) in groups of 64 keys inside each tile, the denominator from
// the quantized P (P-Reordering) or the raw P, O = alpha O + P V, out = O / denominator;
// the queries are the last sq positions of the sequence (bottom-right causal).
//
// A decode step reads the whole cache for very little arithmetic, so it must spread the
// keys over the GPU. The running max makes a plain split-K inexact -- P of a tile is
// quantized relative to the max through that tile, not a split's local max. Here the max
// is known before any P is formed:
//   pass 1  (persistent: each CTA a run of (batch, kv head, key tile) units, K tiles in a
//           3-stage TMA ring) raw scores q.k for the G = hq / hkv query heads x sq
//           positions of the group (R rows) and each tile's per-row max, into the
//           workspace;
//   pass 2  (grid: splits of split_tiles tiles x (batch, kv head), V tiles in a 3-stage
//           ring; split_tiles from the shape, one wave of CTAs) every split starts from
//           the exact running max before its first tile (a max over the pass-1 tile maxima),
//           so each tile's P, its HiF4 codes and its alpha are the sequential ones; the
//           split's O and denominator are carried exactly as the sequential loop carries
//           them, from the split's first tile;
//   join    (grid: (batch, kv head) x rows) joins the splits: O = sum_s O_s exp2(m_s -
//           m_end), the same for the denominator (what the sequential alphas multiply to, up
//           to fp32 rounding order), out = O / denominator in bf16.
// Three kernels. K and V tiles arrive by TMA (128-byte swizzle, a 3-stage ring per CTA);
// the products q.K^T and P.V run on mma.sync m16n8k16 with register fragments (R <= 32
// rows fill at most two m-blocks, far from a tcgen05 tile), the softmax and HiF4 steps on
// the CUDA cores. The cache bytes, not the FLOPs, bound a decode step.
#include "common.cuh"
#include "hif4.cuh"

namespace faq {
namespace dec {

constexpr int D = 128;
constexpr int TILE = 128;        // keys per tile (the reference's key chunk)
constexpr int MAX_ROWS = 32;     // G * sq
constexpr int THREADS = 256;
constexpr int STAGES = 3;        // K (pass 1) and V (pass 2) tiles in flight per CTA
// tiles per pass-2 split: one wave of the 2 resident CTAs per SM of a 148-SM B200 over
// all (batch, kv head) pairs, 2 .. 16 tiles (a function of the shape only, so the
// workspace size is too)
inline int64_t split_tiles_for(int64_t ntiles, int64_t bh) {
  const int64_t t = (ntiles * bh + 295) / 296;
  return t < 2 ? 2 : (t > 16 ? 16 : t);
}

struct Params {
  const __nv_bfloat16 *q, *k, *v;
  int64_t qb, qh, qs, kb, kh, ks, vb, vh, vs;
  int batch, hq, hkv, group, sq, sk, rows, rows8, ntiles, nsplits, split_tiles;
  float scale_log2;  // scale * log2(e)
  int p_levels;      // 0: P not quantized
  int raw_normalizer;
  __nv_bfloat16* out;
  int64_t ob, os, oh;
  float* scores;     // [B*hkv][rows][ntiles*TILE] raw q.k
  float* tmax;       // [B*hkv][rows][ntiles] raw per-tile row max (-inf: fully masked)
  float* part_o;     // [B*hkv][nsplits][rows][D]
  float* part_l;     // [B*hkv][nsplits][rows]
  float* part_m;     // [B*hkv][nsplits][rows] log2-domain running max after the split
};

// workspace sections, each rounded up to 16 floats (64 bytes) so every section starts aligned
__host__ __device__ inline int64_t round16(int64_t n) { return (n + 15) / 16 * 16; }
__host__ __device__ inline size_t workspace_floats(int64_t bh, int64_t rows, int64_t ntiles, int64_t nsplits) {
  return static_cast<size_t>(round16(bh * rows * ntiles * TILE) + round16(bh * rows * ntiles) +
                             round16(bh * nsplits * rows * D) + 2 * round16(bh * nsplits * rows));
}

// row r of a group: query head g = r / sq, query position i = r % sq; its last visible key
__device__ __forceinline__ int last_key(const Params& p, int r) { return p.sk - p.sq + (r % p.sq); }


// ---------------------------------------------------------------- pass 1
// K and V tiles arrive by TMA in the 128-byte-swizzled layout: channels 64 h .. 64 h + 63
// of key kk form the 128-byte row kk of region h (16 KB), whose 16-byte unit u (channels
// 8u .. 8u + 7) sits at unit position u ^ (kk % 8). Keys past the cache end are zeros.
constexpr int TILE_BYTES = TILE * D * 2;     // 32 KB
constexpr int REGION_BYTES = TILE * 128;      // 16 KB
__device__ __forceinline__ const unsigned char* sw_unit(const unsigned char* tile, int kk, int channel) {
  return tile + (channel >> 6) * REGION_BYTES + kk * 128 + ((((channel & 63) >> 3) ^ (kk & 7)) << 4);
}

// Scores of the tile on the tensor cores with mma.sync m16n8k16 (bf16 in, fp32
// accumulate): A = the group's q rows (16 per m-block, rows past p.rows zero) held as
// fragments in registers for the whole run, B = K^T read straight from the swizzled tile
// (lane l of an 8-key block reads 2 channels of key l / 4: one 32-bit load, the 8 keys on
// different banks). Warp w covers keys 16 w .. 16 w + 15 (two n-blocks). The decode pass
// is bound by reading the cache; the products are a small part of its time, so the
// register-fragment MMA serves without tensor memory.
constexpr int MBLK = MAX_ROWS / 16;  // m-blocks of 16 rows
// q fragments of m-block mb for the kv head (b, hk): row g = lane / 4 and g + 8, channels
// 16 ks + 2 (lane % 4) (+1) and + 8 (the m16n8k16 A layout)
__device__ __forceinline__ void load_q_frags(const Params& p, int b, int hk, int mb, int lane, uint32_t (&qa)[8][4]) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = mb * 16 + g + 8 * h;
    const __nv_bfloat16* qrow = nullptr;
    if (r < p.rows)
      qrow = p.q + b * p.qb + static_cast<int64_t>(hk * p.group + r / p.sq) * p.qh + static_cast<int64_t>(r % p.sq) * p.qs;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qa[ks][h] = qrow ? *reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 2 * t) : 0u;
      qa[ks][2 + h] = qrow ? *reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 8 + 2 * t) : 0u;
    }
  }
}
__device__ __forceinline__ void score_tile_mma(const Params& p, const unsigned char* s_k, const uint32_t (&qa)[8][4],
                                               int mb, float* s_s, int tile, int warp, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int nb = 0; nb < 2; ++nb) {
    const int kk = warp * 16 + nb * 8 + g;  // this lane's key for the B fragments
    float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const uint32_t b0 = *reinterpret_cast<const uint32_t*>(sw_unit(s_k, kk, 16 * ks) + 4 * t);
      const uint32_t b1 = *reinterpret_cast<const uint32_t*>(sw_unit(s_k, kk, 16 * ks + 8) + 4 * t);
      mma_bf16_16816(c, qa[ks], b0, b1);
    }
    // c[0], c[1]: row g, keys 2t, 2t + 1 of the block; c[2], c[3]: row g + 8
    const int k0 = warp * 16 + nb * 8 + 2 * t;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mb * 16 + g + 8 * h;
      if (r < p.rows) {
        const int lk = last_key(p, r);
        s_s[r * TILE + k0] = (tile * TILE + k0 <= lk) ? c[2 * h] : -INFINITY;
        s_s[r * TILE + k0 + 1] = (tile * TILE + k0 + 1 <= lk) ? c[2 * h + 1] : -INFINITY;
      }
    }
  }
}

// Dynamic shared memory (base rounded up to 1024 bytes for the swizzled TMA tiles):
// STAGES K tiles, the group's q rows in fp32, the tile's scores (rows8 = rows rounded up
// to 8), STAGES mbarriers.
constexpr int BAR_BYTES = 64;
inline size_t scores_smem(int rows8) {
  return 1024 + static_cast<size_t>(STAGES) * TILE_BYTES + static_cast<size_t>(rows8) * TILE * 4 + BAR_BYTES;
}

__global__ void __launch_bounds__(THREADS, 2) decode_scores_kernel(const __grid_constant__ CUtensorMap tmap_k,
                                                                    Params p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* s_kbuf =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* s_s = reinterpret_cast<float*>(s_kbuf + STAGES * TILE_BYTES);  // [rows8][TILE]
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_s + p.rows8 * TILE);    // [STAGES]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // units u = bh * ntiles + tile, a contiguous run per CTA (one q load per kv head)
  const int64_t units = static_cast<int64_t>(p.batch) * p.hkv * p.ntiles;
  const int64_t per = (units + gridDim.x - 1) / gridDim.x;
  const int64_t u0 = blockIdx.x * per, u1 = std::min<int64_t>(units, u0 + per);
  if (u0 >= u1) return;
  if (tid == 0) {
    for (int s0 = 0; s0 < STAGES; ++s0) mbar_init(smem_addr(&bars[s0]), 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmap_k);
  }
  __syncthreads();
  // launched early behind the previous kernel of the stream (which may have written q or
  // the cache): everything above touched only shared memory and the tensor map
  grid_dependency_wait();
  allow_dependent_launch();  // pass 2 may start setting up on SMs this pass leaves
  auto load_k = [&](int64_t u, int stage) {  // thread 0: the tile as two 64-channel boxes
    const int tile = static_cast<int>(u % p.ntiles), bh = static_cast<int>(u / p.ntiles);
    const uint32_t bar = smem_addr(&bars[stage]);
    mbar_arrive_expect_tx(bar, TILE_BYTES);
    for (int c = 0; c < 2; ++c)
      tma_load_4d(smem_addr(s_kbuf + stage * TILE_BYTES + c * REGION_BYTES), &tmap_k, bar, c * 64, tile * TILE,
                  bh % p.hkv, bh / p.hkv);
  };
  if (tid == 0)
    for (int s0 = 0; s0 < STAGES - 1; ++s0)
      if (u0 + s0 < u1) load_k(u0 + s0, s0);
  int cur_bh = -1;
  uint32_t qa[MBLK][8][4];
  int64_t u = u0;
  for (; u < u1; ++u) {
    const int it = static_cast<int>(u - u0);
    __syncthreads();  // the stage refilled below and s_s were last read by the previous unit
    if (tid == 0 && u + STAGES - 1 < u1) load_k(u + STAGES - 1, (it + STAGES - 1) % STAGES);
    const int tile = static_cast<int>(u % p.ntiles), bh = static_cast<int>(u / p.ntiles);
    const int b = bh / p.hkv, hk = bh % p.hkv;
    if (bh != cur_bh) {  // CTA-uniform: the q fragments of the new kv head
      cur_bh = bh;
#pragma unroll
      for (int mb = 0; mb < MBLK; ++mb)
        if (mb * 16 < p.rows) load_q_frags(p, b, hk, mb, lane, qa[mb]);
    }
    // this unit's K tile landed (bounded; a timeout ends the CTA's run after a drain)
    if (!__syncthreads_and(mbar_wait(smem_addr(&bars[it % STAGES]), (it / STAGES) & 1))) {
      if (tid == 0) {
        trace_timeout(40, it);
        for (int64_t v2 = u; v2 < std::min<int64_t>(u1, u + STAGES); ++v2) {  // copies still in flight
          const int iv = static_cast<int>(v2 - u0);
          mbar_wait(smem_addr(&bars[iv % STAGES]), (iv / STAGES) & 1);
        }
      }
      break;
    }
    const unsigned char* s_k = s_kbuf + (it % STAGES) * TILE_BYTES;
#pragma unroll
    for (int mb = 0; mb < MBLK; ++mb)
      if (mb * 16 < p.rows) score_tile_mma(p, s_k, qa[mb], mb, s_s, tile, warp, lane);
    __syncthreads();
    float* dst = p.scores + (static_cast<int64_t>(bh) * p.rows) * (p.ntiles * TILE) + static_cast<int64_t>(tile) * TILE;
    for (int i = tid; i < p.rows * TILE; i += THREADS) {
      const int r = i / TILE, kk = i % TILE;
      dst[static_cast<int64_t>(r) * (p.ntiles * TILE) + kk] = s_s[i];
    }
    // per-row tile max: one warp per row
    for (int r = warp; r < p.rows; r += THREADS / 32) {
      float m = -INFINITY;
      for (int kk = lane; kk < TILE; kk += 32) m = fmaxf(m, s_s[r * TILE + kk]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) p.tmax[(static_cast<int64_t>(bh) * p.rows + r) * p.ntiles + tile] = m;
    }
  }
}

// ---------------------------------------------------------------- pass 2
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}


// Dynamic shared memory: STAGES V tiles (the next ones arrive by TMA while this one is
// multiplied), P of the tile in bf16 and per-row scalars for the rows rounded up to a
// multiple of 16 (the m-blocks), the mbarriers.
constexpr int PS = TILE + 8;  // P row stride (elements): 16 bytes of padding spread the rows over the banks
inline size_t pv_smem(int rows) {
  const size_t prow = 16 * static_cast<size_t>((rows + 15) / 16);
  return 1024 + static_cast<size_t>(STAGES) * TILE_BYTES + prow * PS * 2 + 3 * prow * 4 + 8 + BAR_BYTES;
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// P.V on the tensor cores with mma.sync m16n8k16: A = P of the tile (bf16, rows past
// p.rows zero) from shared memory, B = V from the swizzled tile through ldmatrix.trans
// (keys are the reduction dimension). Warp w owns output channels 16 w .. 16 w + 15 (two
// n-blocks) for every row and keeps them in registers across the split, rescaled by
// alpha per tile, so the warps never combine partial sums.
__global__ void __launch_bounds__(THREADS, 2) decode_pv_kernel(const __grid_constant__ CUtensorMap tmap_v, Params p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* s_vbuf =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __nv_bfloat16* s_p = reinterpret_cast<__nv_bfloat16*>(s_vbuf + STAGES * TILE_BYTES);   // [16 mblk][PS]
  const int prow = 16 * ((p.rows + 15) / 16);                                              // rows of s_p
  float* s_m = reinterpret_cast<float*>(s_p + prow * PS);
  float* s_alpha = s_m + prow;
  float* s_sum = s_alpha + prow;
  uint64_t* bars = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(s_sum + prow) + 7) & ~uintptr_t(7));
  const int split = blockIdx.x, bh = blockIdx.y;
  const int b = bh / p.hkv, hk = bh % p.hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t0 = split * p.split_tiles, t1 = min(p.ntiles, t0 + p.split_tiles);
  const float* tmax = p.tmax + static_cast<int64_t>(bh) * p.rows * p.ntiles;
  if (tid == 0) {
    for (int s0 = 0; s0 < STAGES; ++s0) mbar_init(smem_addr(&bars[s0]), 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmap_v);
  }
  __syncthreads();
  auto prefetch_v = [&](int t, int buf) {  // thread 0: the tile as two 64-channel boxes
    const uint32_t bar = smem_addr(&bars[buf]);
    mbar_arrive_expect_tx(bar, TILE_BYTES);
    for (int c = 0; c < 2; ++c)
      tma_load_4d(smem_addr(s_vbuf + buf * TILE_BYTES + c * REGION_BYTES), &tmap_v, bar, c * 64, t * TILE, hk, b);
  };
  if (tid == 0)
    for (int s0 = 0; s0 < STAGES - 1; ++s0)
      if (t0 + s0 < t1) prefetch_v(t0 + s0, s0);
  // rows p.rows .. prow - 1 of P and of the per-row scalars stay zero
  for (int i = p.rows * PS + tid; i < prow * PS; i += THREADS) s_p[i] = __float2bfloat16_rn(0.0f);
  for (int i = p.rows + tid; i < prow; i += THREADS) s_m[i] = s_alpha[i] = s_sum[i] = 0.0f;
  // Everything above touches only shared memory and the V cache, which pass 1 does not
  // write: it overlaps pass 1's last tiles. The scores and tile maxima are read below.
  grid_dependency_wait();
  allow_dependent_launch();
  // running max before the split (log2 domain): max over the earlier tiles' maxima
  for (int r = warp; r < p.rows; r += THREADS / 32) {
    float m = -INFINITY;
#pragma unroll 4
    for (int t = lane; t < t0; t += 32) m = fmaxf(m, tmax[r * p.ntiles + t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) s_m[r] = m == -INFINITY ? -INFINITY : __fmul_rn(m, p.scale_log2);
  }
  const int g = lane >> 2, tq = lane & 3;
  const int mblocks = prow / 16;  // 1 or 2
  float acc[MBLK][2][4];          // [m-block][n-block][fragment]
#pragma unroll
  for (int mb = 0; mb < MBLK; ++mb)
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[mb][nb][c] = 0.0f;
  float l_row = 0.0f;  // thread tid < rows carries row tid's denominator
  __syncthreads();
  const float* sc = p.scores + static_cast<int64_t>(bh) * p.rows * (p.ntiles * TILE);
  // The P work of a tile: 8-lane groups of 8 keys x one row's 64-key HiF4 group, at most
  // two groups per lane (rows <= 32); each lane's scores (and row tid's tile max) for the
  // next tile are loaded while this tile is multiplied.
  const int ngroups = p.rows * (TILE / 64);
  float4 nxt[2][2];
  float tm_next = -INFINITY;
  auto fetch = [&](int t) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int grp = warp * 4 + q * 4 * (THREADS / 32) + (lane >> 3);
      if (grp < ngroups && t < t1) {
        const float* srow = sc + static_cast<int64_t>(grp / (TILE / 64)) * (p.ntiles * TILE) + t * TILE +
                            (grp % (TILE / 64)) * 64 + (lane & 7) * 8;
        nxt[q][0] = *reinterpret_cast<const float4*>(srow);
        nxt[q][1] = *reinterpret_cast<const float4*>(srow + 4);
      }
    }
    if (tid < p.rows && t < t1) tm_next = tmax[tid * p.ntiles + t];
  };
  fetch(t0);
  bool ok = true;
  for (int t = t0; t < t1; ++t) {
    float4 cur[2][2] = {{nxt[0][0], nxt[0][1]}, {nxt[1][0], nxt[1][1]}};
    const float tm_cur = tm_next;
    fetch(t + 1);
    const int buf = (t - t0) % STAGES;
    if (tid == 0 && t + STAGES - 1 < t1) prefetch_v(t + STAGES - 1, (t - t0 + STAGES - 1) % STAGES);  // tile t-1's stage
    // new running max and alpha per row (the reference's order: max includes this tile)
    if (tid < p.rows) {
      const float tm = tm_cur;
      const float m_old = s_m[tid];
      const float m_new = fmaxf(m_old, tm == -INFINITY ? -INFINITY : __fmul_rn(tm, p.scale_log2));
      const float m_use = m_new == -INFINITY ? 0.0f : m_new;
      s_alpha[tid] = m_old == -INFINITY ? 0.0f : ex2(__fsub_rn(m_old, m_use));
      s_m[tid] = m_new;
      s_sum[tid] = 0.0f;
    }
    __syncthreads();
    // P = exp2(s c - m), HiF4 per 64 keys: 8 lanes x 8 keys per group, four groups per warp
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int g0 = warp * 4 + q * 4 * (THREADS / 32);
      if (g0 >= ngroups) break;  // warp-uniform
      const int grp = g0 + (lane >> 3);
      const bool live = grp < ngroups;
      const int r = live ? grp / (TILE / 64) : 0, half = grp % (TILE / 64);
      const int kk0 = half * 64 + (lane & 7) * 8;
      const float m = s_m[r];
      const float m_use = m == -INFINITY ? 0.0f : m;
      float v8[8];
      const float4 sa = live ? cur[q][0] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      const float4 sb = live ? cur[q][1] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      const float sv[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) v8[i] = sv[i] == -INFINITY ? 0.0f : ex2(__fmaf_rn(sv[i], p.scale_log2, -m_use));
      float raw = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) raw = __fadd_rn(raw, v8[i]);
      float q8[8];
      if (p.p_levels != 0) {
        uint32_t meta;
        hif4_quant8(v8, p.p_levels, q8, meta);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) q8[i] = bf16_round(v8[i]);  // P enters the PV product as bf16
      }
      float qs = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) qs = __fadd_rn(qs, q8[i]);
      float contrib = (p.raw_normalizer || p.p_levels == 0) ? raw : qs;
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) contrib = __fadd_rn(contrib, __shfl_xor_sync(0xffffffffu, contrib, o));
      if (live) {
#pragma unroll
        for (int i = 0; i < 8; ++i) s_p[r * PS + kk0 + i] = __float2bfloat16_rn(q8[i]);  // exact for HiF4
        if ((lane & 7) == 0) atomicAdd(&s_sum[r], contrib);
      }
    }
    // this tile's V landed (bounded; a timeout ends the split after a drain)
    if (!__syncthreads_and(mbar_wait(smem_addr(&bars[buf]), ((t - t0) / STAGES) & 1))) {
      if (tid == 0) {
        trace_timeout(41, t);
        for (int t2 = t; t2 < min(t1, t + STAGES); ++t2)  // copies still in flight
          mbar_wait(smem_addr(&bars[(t2 - t0) % STAGES]), ((t2 - t0) / STAGES) & 1);
      }
      ok = false;
      break;
    }
    if (tid < p.rows) l_row = __fadd_rn(__fmul_rn(s_alpha[tid], l_row), s_sum[tid]);
    const unsigned char* vt = s_vbuf + buf * TILE_BYTES;
    // O = alpha O + P V for this warp's 16 channels
#pragma unroll
    for (int mb = 0; mb < MBLK; ++mb) {
      if (mb < mblocks) {
        const float a_lo = s_alpha[mb * 16 + g], a_hi = s_alpha[mb * 16 + g + 8];
#pragma unroll
        for (int nb = 0; nb < 2; ++nb) {
          acc[mb][nb][0] *= a_lo;
          acc[mb][nb][1] *= a_lo;
          acc[mb][nb][2] *= a_hi;
          acc[mb][nb][3] *= a_hi;
        }
      }
    }
    // ldmatrix.trans rows: matrix m = lane / 8 holds keys 8 (m % 2) + (lane % 8) of the
    // k-step and channels 16 warp + 8 (m / 2) .. + 7
    const int lm = lane >> 3, li = lane & 7;
#pragma unroll 2
    for (int ks = 0; ks < TILE / 16; ++ks) {
      uint32_t bv[4];
      ldmatrix_x4_trans(bv, smem_addr(sw_unit(vt, 16 * ks + 8 * (lm & 1) + li, 16 * warp + 8 * (lm >> 1))));
#pragma unroll
      for (int mb = 0; mb < MBLK; ++mb) {
        if (mb < mblocks) {
          const __nv_bfloat16* prow0 = s_p + (mb * 16 + g) * PS + 16 * ks + 2 * tq;
          uint32_t a[4];
          a[0] = *reinterpret_cast<const uint32_t*>(prow0);
          a[1] = *reinterpret_cast<const uint32_t*>(prow0 + 8 * PS);
          a[2] = *reinterpret_cast<const uint32_t*>(prow0 + 8);
          a[3] = *reinterpret_cast<const uint32_t*>(prow0 + 8 * PS + 8);
          mma_bf16_16816(acc[mb][0], a, bv[0], bv[1]);
          mma_bf16_16816(acc[mb][1], a, bv[2], bv[3]);
        }
      }
    }
    __syncthreads();  // P, the scalars and this V buffer are rewritten next tile
  }
  if (!ok) return;  // the device status records the timeout; the partial results are not written
  const int64_t base = (static_cast<int64_t>(bh) * p.nsplits + split) * p.rows;
  // acc[mb][nb]: rows 16 mb + g (fragments 0, 1) and + 8 (2, 3), channels 16 warp + 8 nb + 2 tq, + 1
#pragma unroll
  for (int mb = 0; mb < MBLK; ++mb) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mb * 16 + g + 8 * h;
      if (mb < mblocks && r < p.rows) {
#pragma unroll
        for (int nb = 0; nb < 2; ++nb)
          *reinterpret_cast<float2*>(p.part_o + (base + r) * D + 16 * warp + 8 * nb + 2 * tq) =
              make_float2(acc[mb][nb][2 * h], acc[mb][nb][2 * h + 1]);
      }
    }
  }
  if (tid < p.rows) {
    p.part_l[base + tid] = l_row;
    p.part_m[base + tid] = s_m[tid];
  }
}

// ---------------------------------------------------------------- join
// One CTA of 4 x 128 threads per (batch, kv head, row): group g adds splits g, g + 4, ...
// (the splits' loads are independent), then the four partial sums meet in shared memory:
// O = sum_s O_s exp2(m_s - m_end), the same for the denominator (what the sequential
// alphas multiply to, up to fp32 rounding order), out = O / denominator in bf16.
__global__ void __launch_bounds__(4 * D) decode_combine_kernel(Params p) {
  __shared__ float s_o[4][D], s_l[4];
  grid_dependency_wait();  // launched early, behind pass 2
  allow_dependent_launch();  // the next call's pass 1 may set up (it writes no part_*)
  const int bh = blockIdx.x, r = blockIdx.y, dd = threadIdx.x % D, grp = threadIdx.x / D;
  const int b = bh / p.hkv, hk = bh % p.hkv;
  const int64_t base = static_cast<int64_t>(bh) * p.nsplits * p.rows;
  const float m_end = p.part_m[base + static_cast<int64_t>(p.nsplits - 1) * p.rows + r];
  const float m_use = m_end == -INFINITY ? 0.0f : m_end;
  float o = 0.0f, l = 0.0f;
#pragma unroll 4
  for (int sp = grp; sp < p.nsplits; sp += 4) {
    const float ms = p.part_m[base + static_cast<int64_t>(sp) * p.rows + r];
    const float f = ms == -INFINITY ? 0.0f : ex2(__fsub_rn(ms, m_use));
    o = __fmaf_rn(p.part_o[(base + static_cast<int64_t>(sp) * p.rows + r) * D + dd], f, o);
    l = __fmaf_rn(p.part_l[base + static_cast<int64_t>(sp) * p.rows + r], f, l);
  }
  s_o[grp][dd] = o;
  if (dd == 0) s_l[grp] = l;
  __syncthreads();
  if (grp == 0) {
    o = __fadd_rn(__fadd_rn(s_o[0][dd], s_o[1][dd]), __fadd_rn(s_o[2][dd], s_o[3][dd]));
    l = __fadd_rn(__fadd_rn(s_l[0], s_l[1]), __fadd_rn(s_l[2], s_l[3]));
    const float y = l > 0.0f ? __fdiv_rn(o, l) : 0.0f;
    const int g = r / p.sq, i_pos = r % p.sq;
    p.out[b * p.ob + static_cast<int64_t>(i_pos) * p.os + static_cast<int64_t>(hk * p.group + g) * p.oh + dd] =
        __float2bfloat16_rn(y);
  }
}

}  // namespace dec
}  // namespace faq

namespace faq {
static int decode_setup(dec::Params& p, const void* q, const void* k, const void* v, int64_t batch, int64_t hq,
                        int64_t hkv, int64_t sq, int64_t sk, int d, int64_t qb, int64_t qh, int64_t qs, int64_t kb,
                        int64_t kh, int64_t ks, int64_t vb, int64_t vh, int64_t vs, float scale, int p_levels,
                        int normalizer_quantized, void* out, int64_t ob, int64_t os, int64_t oh) {
  FAQ_CHECK_ARG(q && k && v && out, "null pointer");
  FAQ_CHECK_ARG(batch > 0 && hq > 0 && hkv > 0 && sq > 0 && sk >= sq, "bad shape (need sk >= sq > 0)");
  FAQ_CHECK_ARG(hq % hkv == 0, "query heads must be divisible by key/value heads");
  if (d != dec::D) return fail(FAQ_ERR_UNSUPPORTED, "head_dim must be 128");
  FAQ_CHECK_ARG((hq / hkv) * sq <= dec::MAX_ROWS, "decode handles at most 32 rows per kv head ((hq / hkv) * sq)");
  FAQ_CHECK_ARG(sk < (int64_t(1) << 30), "cache too long");
  FAQ_CHECK_ARG(p_levels == 0 || p_levels == 123 || p_levels == 12 || p_levels == 13, "p_levels must be 0/123/12/13");
  FAQ_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && qb % 8 == 0 && qh % 8 == 0 && qs % 8 == 0 &&
                    kb % 8 == 0 && kh % 8 == 0 && ks % 8 == 0 && vb % 8 == 0 && vh % 8 == 0 && vs % 8 == 0,
                "Q/K/V must be 16-byte aligned with strides multiple of 8");
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.qb = qb; p.qh = qh; p.qs = qs; p.kb = kb; p.kh = kh; p.ks = ks; p.vb = vb; p.vh = vh; p.vs = vs;
  p.batch = static_cast<int>(batch);
  p.hq = static_cast<int>(hq);
  p.hkv = static_cast<int>(hkv);
  p.group = static_cast<int>(hq / hkv);
  p.sq = static_cast<int>(sq);
  p.sk = static_cast<int>(sk);
  p.rows = p.group * p.sq;
  p.rows8 = (p.rows + 7) / 8 * 8;
  p.ntiles = static_cast<int>((sk + dec::TILE - 1) / dec::TILE);
  p.split_tiles = static_cast<int>(dec::split_tiles_for(p.ntiles, batch * hkv));
  p.nsplits = (p.ntiles + p.split_tiles - 1) / p.split_tiles;
  p.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);
  p.p_levels = p_levels;
  p.raw_normalizer = !normalizer_quantized;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ob = ob; p.os = os; p.oh = oh;
  return FAQ_OK;
}

static int decode_launch(dec::Params& p, float* ws, void* stream) {
  const int64_t bh = static_cast<int64_t>(p.batch) * p.hkv;
  p.scores = ws;
  p.tmax = p.scores + dec::round16(bh * p.rows * p.ntiles * dec::TILE);
  p.part_o = p.tmax + dec::round16(bh * p.rows * p.ntiles);
  p.part_l = p.part_o + dec::round16(bh * p.nsplits * p.rows * dec::D);
  p.part_m = p.part_l + dec::round16(bh * p.nsplits * p.rows);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  FAQ_CHECK_ARG(bh <= 65535, "batch * kv heads must be <= 65535");
  // K and V as [batch][kv head][key][128] with element strides: 64 x 128 boxes, 128-byte
  // swizzle (keys past sk read as zeros)
  CUtensorMap tk, tv;
  {
    const uint32_t box[4] = {64, static_cast<uint32_t>(dec::TILE), 1, 1};
    const uint64_t dims[4] = {static_cast<uint64_t>(dec::D), static_cast<uint64_t>(p.sk), static_cast<uint64_t>(p.hkv),
                              static_cast<uint64_t>(p.batch)};
    const uint64_t ks[3] = {static_cast<uint64_t>(p.ks) * 2, static_cast<uint64_t>(p.kh) * 2,
                            static_cast<uint64_t>(p.kb) * 2};
    const uint64_t vs[3] = {static_cast<uint64_t>(p.vs) * 2, static_cast<uint64_t>(p.vh) * 2,
                            static_cast<uint64_t>(p.vb) * 2};
    int rc = make_tmap(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, p.k, dims, ks, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, p.v, dims, vs, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  const size_t s1 = dec::scores_smem(p.rows8), s2 = dec::pv_smem(p.rows);
  FAQ_CUDA(cudaFuncSetAttribute(dec::decode_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(s1)));
  const int64_t units = bh * p.ntiles;
  const unsigned grid1 = static_cast<unsigned>(std::min<int64_t>(units, static_cast<int64_t>(num_sms()) * 2));
  FAQ_CUDA(cudaFuncSetAttribute(dec::decode_pv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(s2)));
  // All three passes start while the kernel before them drains (programmatic dependent
  // launch) and wait on the device before they read that kernel's results. Pass 1 writes
  // only the scores and tile maxima, which no earlier decode kernel reads once passes 2
  // and 3 of that call have started.
  cudaLaunchAttribute early[1];
  early[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  early[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid1);
  cfg.blockDim = dim3(dec::THREADS);
  cfg.dynamicSmemBytes = s1;
  cfg.stream = st;
  cfg.attrs = early;
  cfg.numAttrs = 1;
  FAQ_CUDA(cudaLaunchKernelEx(&cfg, dec::decode_scores_kernel, tk, p));
  cfg.gridDim = dim3(static_cast<unsigned>(p.nsplits), static_cast<unsigned>(bh));
  cfg.dynamicSmemBytes = s2;
  FAQ_CUDA(cudaLaunchKernelEx(&cfg, dec::decode_pv_kernel, tv, p));
  cfg.gridDim = dim3(static_cast<unsigned>(bh), static_cast<unsigned>(p.rows));
  cfg.blockDim = dim3(4 * dec::D);
  cfg.dynamicSmemBytes = 0;
  FAQ_CUDA(cudaLaunchKernelEx(&cfg, dec::decode_combine_kernel, p));

  return launch_status("hif4 decode kernels");
}
}  // namespace faq

extern "C" size_t faq_hif4_decode_workspace_bytes(int64_t batch, int64_t hq, int64_t hkv, int64_t sq, int64_t sk,
                                                  int d) {
  using namespace faq;
  if (batch <= 0 || hkv <= 0 || hq <= 0 || sq <= 0 || sk <= 0 || d != dec::D || hq % hkv) return 0;
  const int64_t rows = (hq / hkv) * sq, ntiles = (sk + dec::TILE - 1) / dec::TILE;
  const int64_t st = dec::split_tiles_for(ntiles, batch * hkv);
  const int64_t nsplits = (ntiles + st - 1) / st;
  return dec::workspace_floats(batch * hkv, rows, ntiles, nsplits) * sizeof(float);
}

extern "C" int faq_hif4_decode_attention(const void* q, const void* k, const void* v, int64_t batch, int64_t hq,
                                         int64_t hkv, int64_t sq, int64_t sk, int d, int64_t qb, int64_t qh,
                                         int64_t qs, int64_t kb, int64_t kh, int64_t ks, int64_t vb, int64_t vh,
                                         int64_t vs, float scale, int p_levels, int normalizer_quantized, void* out,
                                         int64_t ob, int64_t os, int64_t oh, void* workspace, size_t workspace_bytes,
                                         void* stream) {
  using namespace faq;
  dec::Params p;
  int rc = decode_setup(p, q, k, v, batch, hq, hkv, sq, sk, d, qb, qh, qs, kb, kh, ks, vb, vh, vs, scale, p_levels,
                        normalizer_quantized, out, ob, os, oh);
  if (rc) return rc;
  const size_t need = faq_hif4_decode_workspace_bytes(batch, hq, hkv, sq, sk, d);
  FAQ_CHECK_ARG(workspace != nullptr && aligned16(workspace), "workspace must be a 16-byte aligned device buffer");
  FAQ_CHECK_ARG(workspace_bytes >= need, "workspace too small: faq_hif4_decode_workspace_bytes() bytes needed");
  return decode_launch(p, static_cast<float*>(workspace), stream);
}

// ---------------------------------------------------------------- allocation-free decode
// A decode call for callers that cannot allocate device memory: a serving runtime that
// plans all of its memory at start-up and forbids allocations while it serves, or a host
// hot path where cudaMalloc would synchronize the device. Instead of a caller workspace
// the passes use one file-scope scratch array of FAQ_DECODE_STATIC_SCRATCH_BYTES
// (16 MiB, include/faquant_b200.h), which every GPU that loads this library holds until
// the process exits.
//   - The kernels write every scratch word they read within the same call (scores and
//     tile maxima in pass 1, partial results in pass 2), so nothing has to start at zero.
//   - All calls on a device share the one array: calls that may overlap on that GPU
//     (different streams without ordering between them) race; order them on one stream.
//   - The array's device address is looked up (cudaGetSymbolAddress) on the first call on
//     each device, with that device current, and cached; make that first call before
//     any stream capture. The stream must belong to the current device (checked) and to
//     its primary context, the one the runtime API uses. No call allocates through the
//     library; under lazy module loading (CUDA_MODULE_LOADING=LAZY, the default) the
//     first call on a device is when the driver loads this module there, and that load
//     is what places the array in device memory -- so make that first call at start-up.
namespace faq {
namespace dec {
constexpr size_t STATIC_SCRATCH_BYTES = FAQ_DECODE_STATIC_SCRATCH_BYTES;
static_assert(STATIC_SCRATCH_BYTES % 256 == 0, "the scratch array holds whole 256-byte units");
static __device__ __align__(256) float g_static_scratch[STATIC_SCRATCH_BYTES / sizeof(float)];
constexpr int MAX_DEVICES = 64;
static float* g_static_scratch_ptr[MAX_DEVICES] = {};
static std::mutex g_static_scratch_mutex;

static int static_scratch(void* stream, float** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
  if (stream != nullptr) {
    // the cached address is this device's copy of the array: a stream of another device
    // would run the kernels against memory that is not theirs
    int stream_dev = -1;
    err = cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &stream_dev);
    if (err != cudaSuccess) return cuda_fail(err, "cudaStreamGetDevice");
    if (stream_dev != dev)
      return fail(FAQ_ERR_ARG, "the stream belongs to device " + std::to_string(stream_dev) +
                                   ", not to the current device " + std::to_string(dev));
  }
  if (dev < 0 || dev >= MAX_DEVICES) return fail(FAQ_ERR_UNSUPPORTED, "device ordinal beyond 63");
  std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
  if (g_static_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGetSymbolAddress(decode scratch)");
    g_static_scratch_ptr[dev] = static_cast<float*>(ptr);
  }
  *out = g_static_scratch_ptr[dev];
  return FAQ_OK;
}
}  // namespace dec
}  // namespace faq

extern "C" int faq_hif4_decode_attention_static(const void* q, const void* k, const void* v, int64_t batch,
                                                int64_t hq, int64_t hkv, int64_t sq, int64_t sk, int d, int64_t qb,
                                                int64_t qh, int64_t qs, int64_t kb, int64_t kh, int64_t ks,
                                                int64_t vb, int64_t vh, int64_t vs, float scale, int p_levels,
                                                int normalizer_quantized, void* out, int64_t ob, int64_t os,
                                                int64_t oh, void* stream) {
  using namespace faq;
  dec::Params p;
  int rc = decode_setup(p, q, k, v, batch, hq, hkv, sq, sk, d, qb, qh, qs, kb, kh, ks, vb, vh, vs, scale, p_levels,
                        normalizer_quantized, out, ob, os, oh);
  if (rc) return rc;
  const size_t need = faq_hif4_decode_workspace_bytes(batch, hq, hkv, sq, sk, d);
  if (need > dec::STATIC_SCRATCH_BYTES)
    return fail(FAQ_ERR_ARG, "decode needs " + std::to_string(need) +
                                 " bytes of scratch, more than the 16 MiB static array of "
                                 "faq_hif4_decode_attention_static; use faq_hif4_decode_attention with a workspace");
  float* scratch = nullptr;
  rc = dec::static_scratch(stream, &scratch);
  if (rc) return rc;
  return decode_launch(p, scratch, stream);
}
